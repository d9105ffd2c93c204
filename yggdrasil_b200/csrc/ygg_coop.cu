// The latency kernels for small batches (n = 128): C = n / 32 = 4 warps serve one stream, one stream per block.
//
// With a warp per stream, a token's time at small batches is its chain of dependent steps: 5 router rounds of L2 loads
// per layer, the DRAM fetch of the leaf's record, and the layer's arithmetic done by one warp. Here, per layer:
//   - the router resolves 5 tree levels per round: the 31 rows of the 5-level subtree are read by the 4 warps (16 rows
//     per 16-byte load of the block, 2 loads per lane), each warp ballots its rows' decisions, and the decisions meet in
//     shared memory after one barrier; depth 13 takes 3 rounds (5 + 5 + 3) instead of 5;
//   - nothing is prefetched: an L2 prefetch of the last round's 8 candidate records cost more than it saved (a bulk
//     prefetch holds the issuing warp until the copy engine has taken it; one batch-1 token took 3.35 us in the layer
//     wavefront without it, 3.90 us with it split over the warps, 4.18 us from one warp);
//   - the layer's arithmetic is split by the warps: warp w computes row 4 l + w of lane l (the 32-lane record layout
//     keeps each warp's part of a lane in whole 16-byte chunks), the layer-input codes split their chunks over the
//     warps, and the readout rows are split too; the new state meets in shared memory.
// Every integer and f32 operation, and its order, is that of the warp-per-stream kernels (ygg_step.cu), so routes,
// states and logits are the same bits.
//
// Scoring rows (tokens known in advance) at the smallest batches runs the layers of one row as a wavefront instead:
// layer l of token t needs only layer l - 1 of token t and layer l of token t - 1, so one block holds a warp group per
// layer role, each on its own token, ordered by progress counters in shared memory. split_score_kernel (L <= 4) gives
// every routed layer a router group and an update group; pipe_score_kernel (L <= 7) one group per layer. A token of a
// row then costs about one layer's route instead of all layers (c3: 2.8 against 8.6 us per token at batch 1).
#include <cuda_runtime.h>
#include <stdint.h>

#include "ygg_device.cuh"

namespace ygg {

constexpr int kCoopLook = 5;                         // router levels per round
constexpr int kCoopWarps = 4;                        // n / 32
constexpr int kCoopThreads = 32 * kCoopWarps;
constexpr int kCoopBlocksPerSm = 8;                  // 64 registers a thread
constexpr int kCoopClasses = kMaxClasses<32> / kCoopWarps;   // class groups a warp holds

// What one group of 4 warps needs to run a layer: one slot (record, then the table row at its end), its mbarrier, and
// exchange buffers.
struct CoopLayerSmem {
    uint8_t *slot;
    uint32_t slot_bytes;
    uint32_t bar;
    int8_t *zl;
    int *zpart;          // [4 warps][64] layer-input partial dots
    uint32_t *dec;       // [2 parities][2 loads][4 warps] router ballots
};

// Shared memory of a latency-kernel block: the layer buffers, the new state of the current layer, the readout codes of
// every layer (their heads run after the last layer), the NLL's exchange buffers, and `qs`, the stream's whole state
// [L][n] (the step kernel's copy of its input; the score kernel's row state).
struct CoopSmem {
    CoopLayerSmem ly;
    int8_t *qnew, *zq;   // zq: [L][32]
    float *red;          // [4 warps] the warps' logit maxima, [4] the target's logit (score)
    double *exd;         // [8 class groups][32 lanes] exp of the logits (score)
    int8_t *qs;
};

__host__ __device__ constexpr uint32_t coop_slot_bytes(uint32_t rec_max, int n) { return (rec_max + 2 * n + 127) / 128 * 128; }
// slot | bar 16 | zl 64 | zpart 4 x 64 x 4 | dec 16 x 4
__host__ __device__ constexpr uint32_t coop_layer_smem_bytes(uint32_t rec_max, int n) {
    return coop_slot_bytes(rec_max, n) + 16 + 64 + 4 * 64 * 4 + 16 * 4;
}
// layer buffers | qnew n | zq 8 x 32 | red 32 | exd 8 x 32 x 8 | qs
__host__ __device__ constexpr uint32_t coop_smem_bytes(uint32_t rec_max, int n, int qs_bytes) {
    return coop_layer_smem_bytes(rec_max, n) + n + 8 * 32 + 32 + 8 * 32 * 8 + qs_bytes;
}

__device__ __forceinline__ CoopLayerSmem coop_carve_layer(uint8_t *&p, uint32_t rec_max, int n) {
    CoopLayerSmem c;
    c.slot = p;
    c.slot_bytes = coop_slot_bytes(rec_max, n);
    p += c.slot_bytes;
    c.bar = smem_addr(p); p += 16;
    c.zl = (int8_t *)p; p += 64;
    c.zpart = (int *)p; p += 4 * 64 * 4;
    c.dec = (uint32_t *)p; p += 16 * 4;
    return c;
}

__device__ __forceinline__ CoopSmem coop_carve(uint8_t *smem, uint32_t rec_max, int n) {
    CoopSmem c;
    uint8_t *p = smem;
    c.ly = coop_carve_layer(p, rec_max, n);
    c.qnew = (int8_t *)p; p += n;
    c.zq = (int8_t *)p; p += 8 * 32;
    c.red = (float *)p; p += 32;
    c.exd = (double *)p; p += 8 * 32 * 8;
    c.qs = (int8_t *)p;
    return c;
}

// How the 4 warps of a stream meet: the whole block (one stream per block), or a named barrier of 128 threads (one
// warp group of a block that holds several; ids 1-15, id 0 being __syncthreads').
struct BlockBar {
    __device__ __forceinline__ void sync() const { __syncthreads(); }
    __device__ __forceinline__ bool all(bool p) const { return __syncthreads_and(p) != 0; }
};
struct GroupBar {
    uint32_t id;
    __device__ __forceinline__ void sync() const { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
    __device__ __forceinline__ bool all(bool p) const {
        uint32_t r;
        asm volatile(
            "{\n\t.reg .pred a, q;\n\tsetp.ne.u32 a, %1, 0;\n\tbar.red.and.pred q, %2, 128, a;\n\tselp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(r)
            : "r"((uint32_t)p), "r"(id)
            : "memory");
        return r != 0;
    }
};

// The first round without global loads (PRE): `top` holds rows 1-31 of the layer's router (row k + 1 at 128 k, shared
// memory, copied once per block), and t the lane's two thresholds of token x (rows k + 1 for its k = 16 i + 4 warp +
// lane / 8), loaded ahead of time by route_first_thr.
struct RouteFirst {
    const int8_t *top;
    float t[2];
};
__device__ __forceinline__ void route_first_thr(const DevLayer &y, int x, int E, int D, int warp, int lane,
                                                float (&t)[2]) {
    const int nrows = (1 << (D < kCoopLook ? D : kCoopLook)) - 1;
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int k = 16 * i + 4 * warp + lane / 8;
        t[i] = k < nrows ? __ldg(y.thr + (size_t)x * E + k + 1) : 0.0f;
    }
}

// Nothing to overlap with a round's loads (see route_coop's `shadow`).
struct NoShadow {
    __device__ __forceinline__ void operator()() const {}
};

// Router descent of the block's stream (cpu/ygg.cpp:271-280), kCoopLook levels per round. Row k < 31 of a round's
// subtree (heap order under the round's root ix: k = 0 is ix, k = 1-2 its children, ...) is read in load k / 16 by
// warp (k % 16) / 4, row group k % 4 (the 8 lanes 8 g .. 8 g + 7, 16 bytes each). Each lane also reads its row's
// threshold; one ballot per load and warp carries the decisions (bit 8 g), which the warps exchange in `dec`. qb: the
// n new state bytes of the layer below. DT > 0: the depth fixed at compile time (= D), the rounds unrolled. Returns the leaf node index in
// [E, 2E).
//
// shadow() runs in the second round (the first when D <= 5) between the issue of its loads and their use, and after()
// once that round's barrier has passed: work that needs neither the loads nor the decisions hides in their latency.
template <int DT = 0, bool PRE = false, class Bar, class Shadow = NoShadow, class After = NoShadow>
__device__ __forceinline__ int route_coop(const DevLayer &y, int x, int E, int D, const int8_t *qb, float rho,
                                          uint32_t *dec, const Bar &bar, int warp, int lane,
                                          const RouteFirst &pre = RouteFirst{}, const Shadow &shadow = Shadow{},
                                          const After &after = After{}) {
    constexpr int N = 128, LPR = 8;
    const int g = lane / LPR;
    const int8_t *wl = y.w + 16 * (lane % LPR);
    const float *thr_x = y.thr + (size_t)x * E;
    const uint4 qrow = *(const uint4 *)(qb + 16 * (lane % LPR));
    int kk[2], mul[2], add[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int k = 16 * i + 4 * warp + g;
        const int lvl = 31 - __clz(k + 1);
        kk[i] = k;
        mul[i] = 1 << lvl;
        add[i] = k + 1 - (1 << lvl);
    }
    int ix = 1, parity = 0;
    // one round: the lv <= kCoopLook levels under ix, starting at depth d
    auto round = [&](const int d, const int lv) {
        const int nrows = (1 << lv) - 1;
        uint4 v[2];
        float t[2];
        if (PRE && d == 0) {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                v[i] = kk[i] < nrows ? *(const uint4 *)(pre.top + 128 * kk[i] + 16 * (lane % LPR)) : make_uint4(0, 0, 0, 0);
                t[i] = pre.t[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < 2; i++) {
                const int row = ix * mul[i] + add[i];
                v[i] = make_uint4(0, 0, 0, 0);
                t[i] = 0.0f;
                if (kk[i] < nrows) {
                    v[i] = __ldg((const uint4 *)(wl + (size_t)row * N));
                    t[i] = __ldg(thr_x + row);
                }
            }
        }
        const bool hide = d == (D > kCoopLook ? kCoopLook : 0);
        if (hide) shadow();
#pragma unroll
        for (int i = 0; i < 2; i++) {
            int dot = dot16(v[i], qrow, 0);
#pragma unroll
            for (int off = 1; off < LPR; off <<= 1) dot += __shfl_xor_sync(kFull, dot, off);
            const uint32_t bal = __ballot_sync(kFull, __fmul_rn(i2f(dot), rho) > t[i]);
            if (lane == 0) dec[parity * 8 + i * 4 + warp] = bal;
        }
        bar.sync();
        if (hide) after();
        // row k's decision: bit 8 g of dec[load][warp] -> bit k = 16 load + 4 warp + g of one mask
        uint32_t mask = 0;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t b = dec[parity * 8 + j];
            mask |= ((b & 1u) | ((b >> 7) & 2u) | ((b >> 14) & 4u) | ((b >> 21) & 8u)) << (4 * j);
        }
        int k = 0;
#pragma unroll
        for (int j = 0; j < kCoopLook; j++) {
            if (j < lv) {
                const int b = (int)((mask >> k) & 1u);
                ix = 2 * ix + b;
                k = 2 * k + 1 + b;
            }
        }
        parity ^= 1;
    };
    if constexpr (DT > 0) {
#pragma unroll
        for (int d = 0; d < DT; d += kCoopLook) round(d, DT - d < kCoopLook ? DT - d : kCoopLook);
    } else {
        for (int d = 0; d < D; d += kCoopLook) round(d, min(kCoopLook, D - d));
    }
    return ix;
}

struct CoopOut {
    int8_t *q_out;       // where the new state goes: [L][ns] (global memory), or the score kernel's shared [L][n]
    int32_t *routes;     // [L] or null
    int32_t *acc;        // [L][ns] or null
};

// Where a layer's record lands: the slot (record, then the table row at its end) and the mbarrier of its copy.
struct CoopSlot {
    uint8_t *slot;
    uint32_t slot_bytes;
    uint32_t bar;
};

// The layer-input codes zl[k] = clamp(rint((f32(V'_k . qb) * mv[k]) * rho)) (cpu/ygg.cpp:285-296) of layer y from qb,
// the new state of the layer below: warp w dots chunks 2w, 2w+1 into zpart (coop_zl_partial); after a barrier of the
// group, warp 0 adds the 4 partials (coop_zl_finish).
template <int R2T>
__device__ __forceinline__ void coop_zl_partial(const DevModel &m, const DevLayer &y, const int8_t *qb, int *zpart,
                                                int warp, int lane) {
    const int R2P = R2T ? R2T : m.R2P;
    for (int k = lane; k < R2P; k += 32) {
        const int8_t *vk = y.vl + (size_t)k * 16;
        int a = 0;
#pragma unroll
        for (int j = 2 * warp; j < 2 * warp + 2; j++)
            a = dot16(__ldg((const uint4 *)(vk + (size_t)j * R2P * 16)), *(const uint4 *)(qb + 16 * j), a);
        zpart[warp * 64 + k] = a;
    }
}
template <int R2T>
__device__ __forceinline__ void coop_zl_finish(const DevModel &m, const DevLayer &y, float rho, const int *zpart,
                                               int8_t *zl, int warp, int lane) {
    if (warp != 0) return;
    const int R2P = R2T ? R2T : m.R2P;
    for (int k = lane; k < R2P; k += 32) {
        const int a = zpart[k] + zpart[64 + k] + zpart[128 + k] + zpart[192 + k];
        const float zf = __fmul_rn(__fmul_rn(i2f(a), __ldg(y.mv + k)), rho);
        zl[k] = (int8_t)(k < m.R2 ? clampi(cvt_rne(zf), -127, 127) : 0);
    }
}

// The copy of leaf r's record and its table row (for token x) into sl, issued by the calling thread; the slot's
// earlier readers are done (the caller has synchronised with them).
__device__ __forceinline__ void coop_issue_copy(const DevLayer &y, int x, int r, const CoopSlot &sl) {
    constexpr int N = 128;
    const bool has_table = y.table != nullptr;
    uint8_t *trow = sl.slot + sl.slot_bytes - 2 * N;
    fence_proxy_async();
    mbar_expect_tx(sl.bar, y.rec_bytes + (has_table ? 2u * N : 0u));
    bulk_g2s(smem_addr(sl.slot), y.rec + (size_t)r * y.rec_bytes, y.rec_bytes, sl.bar);
    if (has_table)
        bulk_g2s(smem_addr(trow), y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N, 2u * N,
                 sl.bar);
}

// The first half of layer l of one token of a group's stream (4 warps; `bar` joins them): for l > 0 rho, the router
// (PRE: its first round reads `pre`, rows in shared memory and thresholds loaded ahead) and, in the shadow of its
// loads, the layer-input codes into zl (zpart and dec are scratch); then the group's thread 0 starts the copy of the
// chosen record and its table row into `sl` (l = 0: the token's own record). qb: the new state of the layer below
// (shared memory). Returns the leaf r in [0, E).
template <int R2T, bool PRE, class Bar>
__device__ __forceinline__ int coop_route_part(const DevModel &m, int l, int x, const int8_t *qb, int8_t *zl,
                                               int *zpart, uint32_t *dec, const CoopSlot &sl, const Bar &bar,
                                               int warp, int lane, const RouteFirst &pre) {
    constexpr int N = 128, C = kCoopWarps;
    const DevLayer &y = m.layer[l];
    const bool low = l > 0 && (R2T > 0 || m.R2 > 0);
    int r = x;
    float rho = 0.0f;
    if (l > 0) {
        const LaneQ<C> qv = load_q<C>(qb + C * lane);
        rho = rms_rho<N, 32>(qv, y.r2b, y.rms_eps, m.inv_n, lane);
        // the layer-input codes need only the state below and rho: formed while a router round's loads are in flight
        auto zl_part = [&]() {
            if (low) coop_zl_partial<R2T>(m, y, qb, zpart, warp, lane);
        };
        auto zl_sum = [&]() {
            if (low) coop_zl_finish<R2T>(m, y, rho, zpart, zl, warp, lane);
        };
        r = (m.D == 13 ? route_coop<13, PRE>(y, x, m.E, m.D, qb, rho, dec, bar, warp, lane, pre, zl_part, zl_sum)
                       : route_coop<0, PRE>(y, x, m.E, m.D, qb, rho, dec, bar, warp, lane, pre, zl_part, zl_sum)) -
            m.E;
    }
    // -- the record and its table row into the slot (the group's thread 0)
    if (warp == 0 && lane == 0) coop_issue_copy(y, x, r, sl);
    return r;
}

// The second half: the wait (bounded) for the copy into `sl` (its mbarrier's phase `parity`), then row i = 4 lane +
// warp of the update and the readout. zl: the layer-input codes; qold: this layer's old state (shared); qnew: where
// the layer's new state goes (shared); q_out (+ acc_out, route_out = r when not null; QS: q_out is shared memory with
// stride n): the new state's destination; zq: the layer's 32 readout-code bytes (shared). Returns false (every thread
// of the group) if the wait gave up.
template <int BLK, int R, int R2T, bool QS, class Bar>
__device__ __forceinline__ bool coop_update_part(const DevModel &m, int l, int x, int r, const CoopSlot &sl,
                                                 uint32_t parity, const int8_t *zl, const int8_t *qold, int8_t *qnew,
                                                 int8_t *zq, int8_t *q_out, int32_t *acc_out, int32_t *route_out,
                                                 const Bar &bar, int warp, int lane) {
    constexpr int N = 128, C = kCoopWarps;
    const int tid = 32 * warp + lane;
    const int i = C * lane + warp;               // the state coordinate this thread updates
    const int ns = QS ? N : m.ns;
    const DevLayer &y = m.layer[l];
    const bool low = l > 0 && (R2T > 0 || m.R2 > 0);
    const bool has_table = y.table != nullptr;
    const bool ok = mbar_wait_bounded(sl.bar, parity);
    if (!bar.all(ok)) return false;   // every wait ended (or one gave up); zl is ready
    // -- row i = 4 lane + warp: transition, input, layer input, saturation (cpu/ygg.cpp:312-389); the lane's data
    // for its row ii = warp sits in whole chunks of the 32-lane layout
    const uint8_t *rec = sl.slot;
    const int16_t *trow = (const int16_t *)(sl.slot + sl.slot_bytes - 2 * N);
    int acc;
    {
        constexpr int kRowWords = BLK / 2;
        const uint8_t *pa = rec + y.off_a + 16 * lane;
        uint32_t aw[kRowWords];
#pragma unroll
        for (int j = 0; j < kRowWords / 4; j++) {
            const uint4 v = *(const uint4 *)(pa + 512 * (warp * (kRowWords / 4) + j));
            aw[4 * j] = v.x; aw[4 * j + 1] = v.y; aw[4 * j + 2] = v.z; aw[4 * j + 3] = v.w;
        }
        const int blk0 = (i / BLK) * BLK;
        uint32_t qblk[BLK / 4];
        if constexpr (BLK == 8) {
            const uint2 v = *(const uint2 *)(qold + blk0);
            qblk[0] = v.x; qblk[1] = v.y;
        } else {
            const uint4 v = *(const uint4 *)(qold + blk0);
            qblk[0] = v.x; qblk[1] = v.y; qblk[2] = v.z; qblk[3] = v.w;
        }
        int s = 0;
#pragma unroll
        for (int p = 0; p < kRowWords; p++)
            s = (p & 1) ? __dp2a_hi((int)aw[p], (int)qblk[p >> 1], s) : __dp2a_lo((int)aw[p], (int)qblk[p >> 1], s);
        acc = (s + (1 << (m.shift - 1))) >> m.shift;
    }
    if (has_table) {
        acc += trow[i];
    } else {   // factored (cpu/ygg.cpp:339-358): the lane's row ii = warp of F, chunks warp * KP/16 + j
        const int KP = m.KP;
        const uint8_t *pf = rec + y.off_f + 16 * lane;
        const int8_t *v = y.vt + (size_t)x * KP;
        int lt = 0;
        for (int j = 0; j < KP / 16; j++)
            lt = dot16(*(const uint4 *)(pf + 512 * (warp * (KP / 16) + j)), __ldg((const uint4 *)(v + 16 * j)), lt);
        const float su = *(const float *)(rec + y.off_su);
        const float mul = __fmul_rn(su, __ldg(y.mt + i));
        acc += cvt_rne(__fmul_rn(i2f(lt), mul)) + ((const int16_t *)(rec + y.off_cb))[i];
    }
    if (low) {   // (cpu/ygg.cpp:360-377): the lane's row ii = warp of U', chunks warp * R2P/16 + j
        const int R2P = R2T ? R2T : m.R2P;
        const uint8_t *pu = rec + y.off_u + 16 * lane;
        int la = 0;
#pragma unroll
        for (int j = 0; j < (R2T ? R2T / 16 : 4); j++)
            if (R2T || j < R2P / 16)
                la = dot16(*(const uint4 *)(pu + 512 * (warp * (R2P / 16) + j)), *(const uint4 *)(zl + 16 * j), la);
        const float mu = y.mulv ? __ldg(y.mulv + i) : y.layer_input_scale;
        acc += cvt_rne(__fmul_rn(i2f(la), mu));
    }
    if (i >= m.ns) acc = 0;   // padding of a narrower model: held at exactly 0
    const int8_t qn = (int8_t)clampi(acc, -128, 127);
    // the readout reads the new state of every lane: every thread has read the old state and the slot's rows first
    qnew[i] = qn;
    if (!QS && acc_out != nullptr && i < ns) acc_out[i] = acc;
    bar.sync();
    if (tid < ns) q_out[tid] = qnew[tid];
    if (!QS && route_out != nullptr && tid == 0) *route_out = r;
    // -- readout (cpu/ygg.cpp:395-420): warp w takes rows [w R/4, (w + 1) R/4); the lane's word of row rr is
    // P[rr][4 lane .. 4 lane + 3], word rr of its readout data
    {
        constexpr int RW = R / C;
        const uint32_t qw = *(const uint32_t *)(qnew + C * lane);
        const uint32_t *pp = (const uint32_t *)(rec + y.off_p + 16 * lane);
        int myz = 0;
#pragma unroll
        for (int j = 0; j < RW; j++) {
            const int rr = warp * RW + j;
            const uint32_t word = pp[128 * (rr / 4) + rr % 4];
            const int z = __reduce_add_sync(kFull, __dp4a((int)word, (int)qw, 0));
            if (lane == j) myz = z;
        }
        if (lane < RW) {
            const int rr = warp * RW + lane;
            const float mz = y.off_mz != kNone ? *(const float *)(rec + y.off_mz + 4 * rr) : y.readout_scale;
            zq[rr] = (int8_t)clampi(cvt_rne(__fmul_rn(i2f(myz), mz)), -127, 127);
        }
    }
    bar.sync();   // every read of the slot is done before the next copy into it; zq is ready
    return true;
}

// Layer l of one token of a group's stream: both halves, one after the other, through the group's one slot. qnew may
// be qb itself (qb is read only before the record wait).
template <int BLK, int R, int R2T, bool QS, bool PRE = false, class Bar>
__device__ __forceinline__ bool coop_layer(const DevModel &m, const CoopLayerSmem &sm, uint32_t &phase, int l, int x,
                                           const int8_t *qb, const int8_t *qold, int8_t *qnew, int8_t *zq,
                                           int8_t *q_out, int32_t *acc_out, int32_t *route_out, const Bar &bar,
                                           int warp, int lane, const RouteFirst &pre = RouteFirst{}) {
    const CoopSlot sl{sm.slot, sm.slot_bytes, sm.bar};
    const int r = coop_route_part<R2T, PRE>(m, l, x, qb, sm.zl, sm.zpart, sm.dec, sl, bar, warp, lane, pre);
    const uint32_t parity = phase;
    phase ^= 1u;
    return coop_update_part<BLK, R, R2T, QS>(m, l, x, r, sl, parity, sm.zl, qold, qnew, zq, q_out, acc_out, route_out,
                                             bar, warp, lane);
}

// The logits of a token (cpu/ygg.cpp:421-434): head_b, then every layer's head in layer order, for this warp's class
// groups cg = warp + 4 c (classes 32 cg + lane). zq: layer l's readout codes at zq + 32 l. With the layer count fixed,
// the unembedding rows of every layer load together.
template <int R, int LT, int NVT>
__device__ __forceinline__ void coop_heads(const DevModel &m, const int8_t *zq, float (&lg)[kCoopClasses], int warp,
                                           int lane) {
    constexpr int C = kCoopWarps;
    const int L = LT ? LT : m.L;
    const int nv = NVT ? NVT : m.VP / 32;
#pragma unroll
    for (int c = 0; c < kCoopClasses; c++) {
        const int cg = warp + C * c;
        lg[c] = cg < nv ? __ldg(m.head_b + 32 * cg + lane) : 0.0f;
    }
    auto head = [&](const int l) {
        const DevLayer &y = m.layer[l];
        uint32_t zw[R / 4];
#pragma unroll
        for (int j = 0; j < R / 4; j++) zw[j] = *(const uint32_t *)(zq + l * 32 + 4 * j);
#pragma unroll
        for (int c = 0; c < kCoopClasses; c++) {
            const int cg = warp + C * c;
            if (NVT ? (cg < NVT) : (cg < nv)) {
                const int cls = 32 * cg + lane;
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
                const float sc = y.sqv ? __ldg(y.sqv + cls) : y.unembed_scale;
                lg[c] = __fadd_rn(lg[c], __fmul_rn(i2f(a), sc));
            }
        }
    };
    if constexpr (LT > 0) {
#pragma unroll
        for (int l = 0; l < LT; l++) head(l);
    } else {
        for (int l = 0; l < L; l++) head(l);
    }
}

// One token of the block's stream through every layer. The stream's old state is sm.qs ([L][n], shared memory; the
// step kernel copies its input there first, in one pass); the new state goes to o.q_out ([L][ns] in global memory
// for the step kernel; sm.qs itself for the score kernel, QS). lg: the logits of this lane's classes 32 cg + lane for
// the class groups cg = warp + 4 c; every layer's head is added after the last layer (in layer order), so that no
// layer waits on the unembedding's loads. Returns false if the bounded wait for a copy gave up.
template <int BLK, int R, int R2T, int LT, int NVT, bool QS>
__device__ __forceinline__ bool coop_token(const DevModel &m, const CoopSmem &sm, uint32_t &phase, int x,
                                           const CoopOut &o, float (&lg)[kCoopClasses], int warp, int lane) {
    constexpr int N = 128;
    const int L = LT ? LT : m.L, ns = QS ? N : m.ns;
    const BlockBar bar;
#pragma unroll 1
    for (int l = 0; l < L; l++) {
        // the new state of the layer below is in qnew, and this layer's replaces it
        if (!coop_layer<BLK, R, R2T, QS>(m, sm.ly, phase, l, x, sm.qnew, sm.qs + (size_t)l * N, sm.qnew,
                                         sm.zq + l * 32, o.q_out + (size_t)l * ns,
                                         o.acc ? o.acc + (size_t)l * ns : nullptr, o.routes ? o.routes + l : nullptr,
                                         bar, warp, lane))
            return false;
    }
    coop_heads<R, LT, NVT>(m, sm.zq, lg, warp, lane);
    return true;
}

// -log p(y) in f64 over the V classes of the block's stream (cpu/ygg.cpp:513-517), summed in the order of the
// warp-per-stream kernels' nll_of: lane l adds the exps of its classes 32 cg + l in class-group order, then a butterfly
// over the 32 lanes; the exps come from the warps holding each class group through shared memory. Every thread gets it.
template <int NVT, class Bar>
__device__ __forceinline__ double coop_nll(const DevModel &m, float *red, double *exd, const float (&lg)[kCoopClasses],
                                           int y, const Bar &bar, int warp, int lane) {
    const int nv = NVT ? NVT : m.VP / 32, V = m.V;
    float mx = -__int_as_float(0x7f800000);
#pragma unroll
    for (int c = 0; c < kCoopClasses; c++) {
        const int cg = warp + kCoopWarps * c;
        if (cg < nv && 32 * cg + lane < V) mx = fmaxf(mx, lg[c]);
        if (32 * cg + lane == y) red[kCoopWarps] = lg[c];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
    if (lane == 0) red[warp] = mx;
    bar.sync();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float ly = red[kCoopWarps];
#pragma unroll
    for (int c = 0; c < kCoopClasses; c++) {
        const int cg = warp + kCoopWarps * c;
        if (cg < nv) exd[32 * cg + lane] = 32 * cg + lane < V ? exp((double)lg[c] - (double)mx) : 0.0;
    }
    bar.sync();
    double se = 0.0;
    for (int cg = 0; cg < nv; cg++)
        if (32 * cg + lane < V) se += exd[32 * cg + lane];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) se += __shfl_xor_sync(kFull, se, off);
    return log(se) + (double)mx - (double)ly;
}

// ------------------------------------------------------------------------------------------------ kernels

__device__ __forceinline__ CoopSmem coop_init(uint8_t *smem, uint32_t rec_max) {
    CoopSmem sm = coop_carve(smem, rec_max, 128);
    if (threadIdx.x == 0) {
        mbar_init(sm.ly.bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    return sm;
}

// One decode step of B streams, one stream per block at a time (grid-stride).
template <int BLK, int R, int R2T, int LT, int NVT>
__global__ void __launch_bounds__(kCoopThreads, kCoopBlocksPerSm) coop_step_kernel(
    const __grid_constant__ DevModel m, int B, const int32_t *__restrict__ tokens, const int8_t *state_in,
    int8_t *state_out, float *__restrict__ logits, int32_t *__restrict__ routes, int32_t *__restrict__ acc_out,
    uint32_t rec_max) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const CoopSmem sm = coop_init(smem, rec_max);
    uint32_t phase = 0;
    const int L = m.L, V = m.V, ns = m.ns, nv = NVT ? NVT : m.VP / 32;
    for (int s = blockIdx.x; s < B; s += gridDim.x) {
        const int x = tokens[s];
        if (x < 0 || x >= V) {   // cpu/ygg.cpp:493-495 rejects the whole input; here the stream is skipped
            if (tid == 0) atomicOr(m.status, kStatusBadToken);
            if (logits != nullptr)
                for (int c = tid; c < V; c += kCoopThreads) logits[(size_t)s * V + c] = __int_as_float(0x7fc00000);
            if (state_out != state_in)
                for (int j = tid; j < L * ns; j += kCoopThreads)
                    state_out[(size_t)s * L * ns + j] = state_in[(size_t)s * L * ns + j];
            if (routes != nullptr && tid < L) routes[(size_t)s * L + tid] = -1;
            continue;
        }
        // the stream's old state, every layer in one pass, into the device layout (coordinates past ns are 0)
        const int8_t *q_in = state_in + (size_t)s * L * ns;
        for (int j = tid; j < L * 128; j += kCoopThreads) {
            const int li = j / 128, c = j % 128;
            sm.qs[j] = c < ns ? q_in[(size_t)li * ns + c] : (int8_t)0;
        }
        __syncthreads();
        float lg[kCoopClasses];
        const CoopOut o{state_out + (size_t)s * L * ns, routes ? routes + (size_t)s * L : nullptr,
                        acc_out ? acc_out + (size_t)s * L * ns : nullptr};
        if (!coop_token<BLK, R, R2T, LT, NVT, false>(m, sm, phase, x, o, lg, warp, lane)) {
            if (tid == 0) atomicOr(m.status, kStatusTimeout);
            return;
        }
        if (logits != nullptr) {
#pragma unroll
            for (int c = 0; c < kCoopClasses; c++) {
                const int cg = warp + kCoopWarps * c, cls = 32 * cg + lane;
                if (cg < nv && cls < V) logits[(size_t)s * V + cls] = lg[c];
            }
        }
    }
}

// Rows of T tokens, one row per block at a time: the row's state in shared memory, the f64 NLL of the next token
// summed on chip (cpu/ygg.cpp:513-517).
template <int BLK, int R, int R2T, int LT, int NVT>
__global__ void __launch_bounds__(kCoopThreads, kCoopBlocksPerSm) coop_score_kernel(
    const __grid_constant__ DevModel m, int B, int T, const int32_t *__restrict__ tokens, int8_t *state,
    double *__restrict__ bits, uint32_t rec_max) {
    constexpr int N = 128;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const CoopSmem sm = coop_init(smem, rec_max);
    uint32_t phase = 0;
    const int L = m.L, V = m.V, ns = m.ns;
    for (int s = blockIdx.x; s < B; s += gridDim.x) {
        const int32_t *tok = tokens + (size_t)s * T;
        bool bad = false;
        for (int t = tid; t < T; t += kCoopThreads) bad |= tok[t] < 0 || tok[t] >= V;
        if (__syncthreads_or(bad)) {
            if (tid == 0) {
                atomicOr(m.status, kStatusBadToken);
                bits[s] = __longlong_as_double(0x7ff8000000000000LL);
            }
            continue;
        }
        // the row's state into the device layout (n per layer; coordinates past the model's ns are 0)
        for (int j = tid; j < L * N; j += kCoopThreads) {
            const int li = j / N, c = j % N;
            sm.qs[j] = (state != nullptr && c < ns) ? state[((size_t)s * L + li) * ns + c] : (int8_t)0;
        }
        __syncthreads();
        const CoopOut o{sm.qs, nullptr, nullptr};
        double nll = 0.0;
        for (int t = 0; t + 1 < T; t++) {
            float lg[kCoopClasses];
            if (!coop_token<BLK, R, R2T, LT, NVT, true>(m, sm, phase, tok[t], o, lg, warp, lane)) {
                if (tid == 0) atomicOr(m.status, kStatusTimeout);
                return;
            }
            nll += coop_nll<NVT>(m, sm.red, sm.exd, lg, tok[t + 1], BlockBar{}, warp, lane);
        }
        if (tid == 0) bits[s] = nll / 0.69314718055994530942;
        if (state != nullptr)
            for (int j = tid; j < L * N; j += kCoopThreads) {
                const int li = j / N, c = j % N;
                if (c < ns) state[((size_t)s * L + li) * ns + c] = sm.qs[j];
            }
        __syncthreads();
    }
}

// Rows of T tokens at the smallest batches, one row per block, the layers as a wavefront (cpu/ygg.cpp:500-519 is the
// sequential loop it reorders). Layer l of token t needs only layer l - 1 of token t (the state it routes on) and
// layer l of token t - 1 (its own old state), so the block's L + 1 warp groups form a pipeline: group g < L runs layer
// g of token after token, and group L forms the logits and the NLL of each token once layer L - 1 has it. The new state
// of layer g goes to group g + 1 through a ring of kPipeHand buffers; the readout codes of a token wait in a ring of
// kPipeRing slots until group L reads them. Each group publishes how many tokens it has finished (`done`, a release
// store after the group's last barrier of the token); a group starts token t once the group below has finished it and
// the groups that read its rings have freed the slots it will write. Nothing else orders the groups, so a token
// costs about the mean time of the slowest layer rather than the sum over the layers. Every operation and every sum's
// order are those of the sequential kernels: the bits match.
constexpr int kPipeRing = 16;   // readout-code slots (tokens between a layer and the NLL group)
constexpr int kPipeHand = 4;    // new-state buffers between two layers

__host__ __device__ constexpr uint32_t pipe_smem_bytes(uint32_t rec_max, int L) {
    // L layer groups' buffers | top rows L x 4096 | hand L x kPipeHand x n | qs L x n | zq ring kPipeRing x L x 32 |
    // red 32 | exd 8 x 32 x 8 | done 8 x 4 | abort 4
    return L * coop_layer_smem_bytes(rec_max, 128) + L * 4096 + L * kPipeHand * 128 + L * 128 + kPipeRing * L * 32 +
           32 + 8 * 32 * 8 + 8 * 4 + 16;
}

__device__ __forceinline__ int ld_acquire_shared(const int *p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_shared(int *p, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}

template <int BLK, int R, int R2T, int LT, int NVT>
__global__ void __launch_bounds__(LT > 0 ? 128 * (LT + 1) : 1024, 1) pipe_score_kernel(
    const __grid_constant__ DevModel m, int B, int T, const int32_t *__restrict__ tokens, int8_t *state,
    double *__restrict__ bits, uint32_t rec_max) {
    constexpr int N = 128;
    extern __shared__ __align__(128) uint8_t smem[];
    const int L = LT ? LT : m.L, V = m.V, ns = m.ns;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int grp = tid >> 7, warp = (tid >> 5) & 3, lane = tid & 31, gtid = tid & 127;
    // carve: every layer group's own buffers, then what the groups share
    uint8_t *p = smem;
    CoopLayerSmem ly{};
    for (int g = 0; g < L; g++) {
        const CoopLayerSmem c = coop_carve_layer(p, rec_max, N);
        if (g == grp) ly = c;
    }
    int8_t *top = (int8_t *)p; p += L * 4096;
    int8_t *hand = (int8_t *)p; p += L * kPipeHand * N;
    int8_t *qs = (int8_t *)p; p += L * N;
    int8_t *zqr = (int8_t *)p; p += kPipeRing * L * 32;
    float *red = (float *)p; p += 32;
    double *exd = (double *)p; p += 8 * 32 * 8;
    int *done = (int *)p; p += 8 * 4;
    int *abort_flag = (int *)p;
    if (grp < L && gtid == 0) {
        mbar_init(ly.bar, 1);
        fence_mbar_init();
    }
    {   // rows 1 .. 2^min(5, D) - 1 of every routed layer's router, for the first round of each of its tokens
        const int nrows = (1 << (m.D < kCoopLook ? m.D : kCoopLook)) - 1;
        for (int j = tid; j < L * 256; j += nthr) {
            const int g = j >> 8, c = j & 255;
            if (g > 0 && c < 8 * nrows)
                *(uint4 *)(top + 4096 * g + 16 * c) = __ldg((const uint4 *)(m.layer[g].w + N + 16 * c));
        }
    }
    __syncthreads();
    const GroupBar bar{1u + (uint32_t)grp};
    const bool routed = grp > 0 && grp < L;
    uint32_t phase = 0;
    for (int s = blockIdx.x; s < B; s += gridDim.x) {
        const int32_t *tok = tokens + (size_t)s * T;
        bool bad = false;
        for (int t = tid; t < T; t += nthr) bad |= tok[t] < 0 || tok[t] >= V;
        if (__syncthreads_or(bad)) {
            if (tid == 0) {
                atomicOr(m.status, kStatusBadToken);
                bits[s] = __longlong_as_double(0x7ff8000000000000LL);
            }
            continue;
        }
        for (int j = tid; j < L * N; j += nthr) {
            const int li = j / N, c = j % N;
            qs[j] = (state != nullptr && c < ns) ? state[((size_t)s * L + li) * ns + c] : (int8_t)0;
        }
        if (tid < 8) done[tid] = 0;
        if (tid == 0) *abort_flag = 0;
        __syncthreads();
        double nll = 0.0;
        bool ok = true;
        // the first router round's thresholds need only the token: each token's are loaded one token ahead
        float tn[2] = {0.0f, 0.0f};
        if (routed && T > 1) route_first_thr(m.layer[grp], tok[0], m.E, m.D, warp, lane, tn);
        for (int t = 0; t + 1 < T; t++) {
            const RouteFirst pre{top + 4096 * grp, {tn[0], tn[1]}};
            if (routed && t + 2 < T) route_first_thr(m.layer[grp], tok[t + 1], m.E, m.D, warp, lane, tn);
            // wait (the group's thread 0, bounded) until token t's input is ready and the ring slots it writes are
            // free; the group then agrees on the outcome at its barrier, which also hands the acquired data on
            if (gtid == 0) {
                const long long t0 = clock64();
                for (;;) {
                    const bool in = grp == 0 || ld_acquire_shared(done + grp - 1) > t;
                    const bool hand_free = grp >= L - 1 || ld_acquire_shared(done + grp + 1) > t - kPipeHand;
                    const bool ring_free = grp == L || ld_acquire_shared(done + L) > t - kPipeRing;
                    if (in && hand_free && ring_free) break;
                    if (*(volatile int *)abort_flag != 0 || clock64() - t0 > kWaitCycles) {
                        ok = false;
                        break;
                    }
                }
            }
            if (!bar.all(ok)) {
                ok = false;
                break;
            }
            if (grp < L) {
                const int8_t *qb = grp > 0 ? hand + ((grp - 1) * kPipeHand + t % kPipeHand) * N : nullptr;
                int8_t *qnew = hand + (grp * kPipeHand + t % kPipeHand) * N;
                int8_t *q = qs + grp * N;
                ok = coop_layer<BLK, R, R2T, true, true>(m, ly, phase, grp, tok[t], qb, q, qnew,
                                                         zqr + ((t % kPipeRing) * L + grp) * 32, q, nullptr, nullptr,
                                                         bar, warp, lane, pre);
                if (!ok) break;
            } else {
                float lg[kCoopClasses];
                coop_heads<R, LT, NVT>(m, zqr + (t % kPipeRing) * L * 32, lg, warp, lane);
                nll += coop_nll<NVT>(m, red, exd, lg, tok[t + 1], bar, warp, lane);
            }
            if (gtid == 0) st_release_shared(done + grp, t + 1);
        }
        if (!ok && gtid == 0) atomicExch(abort_flag, 1);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicOr(m.status, kStatusTimeout);
            return;
        }
        if (grp == L && gtid == 0) bits[s] = nll / 0.69314718055994530942;
        if (state != nullptr)
            for (int j = tid; j < L * N; j += nthr) {
                const int li = j / N, c = j % N;
                if (c < ns) state[((size_t)s * L + li) * ns + c] = qs[j];
            }
        __syncthreads();
    }
}

// Rows of T tokens at the smallest batches, L <= 4: the layer wavefront with each routed layer split in two groups.
// The update of layer l at token t needs only the leaf of token t (its record), the layer-input codes and the layer's
// own state after token t - 1, while the route of token t + 1 needs only the state below of token t + 1. So a router
// group (R_l) only routes, token after token, and the update group (U_l) does the rest: it copies the record of the
// leaf R_l left in the token's slot, updates, reads out, and then forms what R_{l+1} and U_{l+1} need from the state it
// just made (rho and the layer-input codes of layer l + 1), while R_l already routes the next tokens (up to
// kSplitSlots ahead). Groups: U_0 (the token layer), R_1, U_1, ..., R_{L-1}, U_{L-1}, then the NLL group: 2L groups
// of 128 threads. Progress counters (doneR, doneU, doneN) order them as in pipe_score_kernel:
//   R_l waits until U_{l-1} has finished the token (its state, rho) and U_l has freed the token's slot;
//   U_l waits until R_l has left the leaf, and until the readers of what it writes (the hand ring, the readout-code
//   ring, the next layer's slot) are far enough;
//   the NLL group waits for U_{L-1}.
// A token then costs about the time of the router's rounds alone. Operations and sums in the same order as the
// sequential kernels: the same bits.
constexpr int kSplitSlots = 3;

// a routed layer's slot for one token: record and table row | mbarrier 16 | layer-input codes 64 | leaf, rho 16
__host__ __device__ constexpr uint32_t split_slot_bytes(uint32_t rec_max) { return coop_slot_bytes(rec_max, 128) + 96; }
__host__ __device__ constexpr uint32_t split_smem_bytes(uint32_t rec_max, int L) {
    // slots: U_0's one, then kSplitSlots per routed layer | zpart 1024 + dec 64 per layer | top rows L x 4096 |
    // hand L x kPipeHand x n | qs L x n | zq ring kPipeRing x L x 32 | red 32 | exd 8 x 32 x 8 | doneR 8 x 4 |
    // doneU 8 x 4 | doneN, abort 16
    return (1 + (L - 1) * kSplitSlots) * split_slot_bytes(rec_max) + L * (1024 + 64) + L * 4096 +
           L * kPipeHand * 128 + L * 128 + kPipeRing * L * 32 + 32 + 8 * 32 * 8 + 8 * 4 + 8 * 4 + 16;
}

template <int BLK, int R, int R2T, int LT, int NVT>
__global__ void __launch_bounds__(LT > 0 ? 256 * LT : 1024, 1) split_score_kernel(
    const __grid_constant__ DevModel m, int B, int T, const int32_t *__restrict__ tokens, int8_t *state,
    double *__restrict__ bits, uint32_t rec_max) {
    constexpr int N = 128, C = kCoopWarps;
    extern __shared__ __align__(128) uint8_t smem[];
    const int L = LT ? LT : m.L, V = m.V, ns = m.ns;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int grp = tid >> 7, warp = (tid >> 5) & 3, lane = tid & 31, gtid = tid & 127;
    // the group's role: U_0 = 0, R_l = 2 l - 1, U_l = 2 l, NLL = 2 L - 1
    const bool is_nll = grp == 2 * L - 1;
    const bool is_r = !is_nll && (grp & 1);
    const int layer = is_r ? (grp + 1) >> 1 : grp >> 1;
    // carve. Slots and their mbarrier phases follow the block's running token count g (the phases carry over from row
    // to row): layer l's slot for token g, and the parity of that use
    const uint32_t cs = coop_slot_bytes(rec_max, N), sb = split_slot_bytes(rec_max);
    uint8_t *slots = smem;
    auto slot_base = [&](int l, int g) {
        return slots + (size_t)sb * (l == 0 ? 0 : 1 + (l - 1) * kSplitSlots + g % kSplitSlots);
    };
    auto slot_of = [&](int l, int g) {
        uint8_t *b = slot_base(l, g);
        return CoopSlot{b, cs, smem_addr(b + cs)};
    };
    auto zl_of = [&](int l, int g) { return (int8_t *)(slot_base(l, g) + cs + 16); };
    auto leaf_of = [&](int l, int g) { return (int *)(slot_base(l, g) + cs + 80); };
    auto rho_of = [&](int l, int g) { return (float *)(slot_base(l, g) + cs + 84); };
    auto parity_of = [&](int l, int g) { return (uint32_t)(l == 0 ? g : g / kSplitSlots) & 1u; };
    uint8_t *p = slots + (size_t)sb * (1 + (L - 1) * kSplitSlots);
    int *zpart = (int *)(p + (size_t)(layer < L ? layer : 0) * (1024 + 64));   // U_l's
    uint32_t *dec = (uint32_t *)((uint8_t *)zpart + 1024);                      // R_l's
    p += (size_t)L * (1024 + 64);
    int8_t *top = (int8_t *)p; p += L * 4096;
    int8_t *hand = (int8_t *)p; p += L * kPipeHand * N;
    int8_t *qs = (int8_t *)p; p += L * N;
    int8_t *zqr = (int8_t *)p; p += kPipeRing * L * 32;
    float *red = (float *)p; p += 32;
    double *exd = (double *)p; p += 8 * 32 * 8;
    int *done_r = (int *)p; p += 8 * 4;
    int *done_u = (int *)p; p += 8 * 4;
    int *done_n = (int *)p;
    int *abort_flag = done_n + 1;
    // every slot's mbarrier (U_0's, then the routed layers')
    for (int j = tid; j < 1 + (L - 1) * kSplitSlots; j += nthr) {
        mbar_init(smem_addr(slots + (size_t)sb * j + cs), 1);
        fence_mbar_init();
    }
    {   // rows 1 .. 2^min(5, D) - 1 of every routed layer's router, for the first round of each of its tokens
        const int nrows = (1 << (m.D < kCoopLook ? m.D : kCoopLook)) - 1;
        for (int j = tid; j < L * 256; j += nthr) {
            const int g = j >> 8, c = j & 255;
            if (g > 0 && c < 8 * nrows)
                *(uint4 *)(top + 4096 * g + 16 * c) = __ldg((const uint4 *)(m.layer[g].w + N + 16 * c));
        }
    }
    __syncthreads();
    const GroupBar bar{1u + (uint32_t)grp};
    int g0 = 0;   // tokens the block has run before this row
    for (int s = blockIdx.x; s < B; s += gridDim.x) {
        const int32_t *tok = tokens + (size_t)s * T;
        bool bad = false;
        for (int t = tid; t < T; t += nthr) bad |= tok[t] < 0 || tok[t] >= V;
        if (__syncthreads_or(bad)) {
            if (tid == 0) {
                atomicOr(m.status, kStatusBadToken);
                bits[s] = __longlong_as_double(0x7ff8000000000000LL);
            }
            continue;
        }
        for (int j = tid; j < L * N; j += nthr) {
            const int li = j / N, c = j % N;
            qs[j] = (state != nullptr && c < ns) ? state[((size_t)s * L + li) * ns + c] : (int8_t)0;
        }
        if (tid < 8) {
            done_r[tid] = 0;
            done_u[tid] = 0;
        }
        if (tid == 0) {
            *done_n = 0;
            *abort_flag = 0;
        }
        __syncthreads();
        double nll = 0.0;
        bool ok = true;
        int inflight = -1;   // (an update group's thread 0) the token whose copy it issued and has not seen land
        float tn[2] = {0.0f, 0.0f};
        if (is_r && T > 1) route_first_thr(m.layer[layer], tok[0], m.E, m.D, warp, lane, tn);
        for (int t = 0; t + 1 < T; t++) {
            const int g = g0 + t;
            const RouteFirst pre{top + 4096 * layer, {tn[0], tn[1]}};
            if (is_r && t + 2 < T) route_first_thr(m.layer[layer], tok[t + 1], m.E, m.D, warp, lane, tn);
            // wait (the group's thread 0, bounded) for this role's inputs and free ring slots; the group agrees at its
            // barrier, which also hands the acquired data to its other threads
            if (gtid == 0) {
                const long long t0 = clock64();
                for (;;) {
                    bool go;
                    if (is_nll) {
                        go = ld_acquire_shared(done_u + L - 1) > t;
                    } else if (is_r) {
                        go = ld_acquire_shared(done_u + layer - 1) > t &&
                             ld_acquire_shared(done_u + layer) > t - kSplitSlots;
                    } else {
                        go = (layer == 0 || ld_acquire_shared(done_r + layer) > t) &&
                             (layer == L - 1 || (ld_acquire_shared(done_r + layer + 1) > t - kPipeHand &&
                                                 ld_acquire_shared(done_u + layer + 1) > t - kSplitSlots)) &&
                             ld_acquire_shared(done_n) > t - kPipeRing;
                    }
                    if (go) break;
                    if (*(volatile int *)abort_flag != 0 || clock64() - t0 > kWaitCycles) {
                        ok = false;
                        break;
                    }
                }
            }
            if (!bar.all(ok)) {
                ok = false;
                break;
            }
            const int x = tok[t];
            if (is_nll) {
                float lg[kCoopClasses];
                coop_heads<R, LT, NVT>(m, zqr + (t % kPipeRing) * L * 32, lg, warp, lane);
                nll += coop_nll<NVT>(m, red, exd, lg, tok[t + 1], bar, warp, lane);
                if (gtid == 0) st_release_shared(done_n, t + 1);
            } else if (is_r) {
                // the route alone (cpu/ygg.cpp:271-280): the state below and rho come from U_{l-1}
                const DevLayer &y = m.layer[layer];
                const int8_t *qb = hand + ((layer - 1) * kPipeHand + t % kPipeHand) * N;
                const float rho = *rho_of(layer, g);
                const int r = (m.D == 13 ? route_coop<13, true>(y, x, m.E, m.D, qb, rho, dec, bar, warp, lane, pre)
                                         : route_coop<0, true>(y, x, m.E, m.D, qb, rho, dec, bar, warp, lane, pre)) -
                              m.E;
                if (gtid == 0) {
                    *leaf_of(layer, g) = r;
                    st_release_shared(done_r + layer, t + 1);
                }
            } else {
                const DevLayer &y = m.layer[layer];
                const CoopSlot sl = slot_of(layer, g);
                // the record of the leaf (the token's own for the token layer) into the token's slot
                if (gtid == 0) {
                    coop_issue_copy(y, x, layer == 0 ? x : *leaf_of(layer, g), sl);
                    inflight = t;
                }
                int8_t *q = qs + layer * N;
                int8_t *qnew = hand + (layer * kPipeHand + t % kPipeHand) * N;
                ok = coop_update_part<BLK, R, R2T, true>(m, layer, x, 0, sl, parity_of(layer, g), zl_of(layer, g), q,
                                                         qnew, zqr + ((t % kPipeRing) * L + layer) * 32, q, nullptr,
                                                         nullptr, bar, warp, lane);
                if (!ok) break;
                inflight = -1;
                if (layer + 1 < L) {   // rho and the layer-input codes of layer + 1 from the new state (cpu/ygg.cpp:248-296)
                    const DevLayer &yn = m.layer[layer + 1];
                    const LaneQ<C> qv = load_q<C>(qnew + C * lane);
                    const float rho = rms_rho<N, 32>(qv, yn.r2b, yn.rms_eps, m.inv_n, lane);
                    if (gtid == 0) *rho_of(layer + 1, g) = rho;
                    if (R2T > 0 || m.R2 > 0) {
                        coop_zl_partial<R2T>(m, yn, qnew, zpart, warp, lane);
                        bar.sync();
                        coop_zl_finish<R2T>(m, yn, rho, zpart, zl_of(layer + 1, g), warp, lane);
                    }
                }
                __syncwarp();   // warp 0 wrote the codes; its lane 0 publishes them
                if (gtid == 0) st_release_shared(done_u + layer, t + 1);
            }
        }
        if (!ok && gtid == 0) atomicExch(abort_flag, 1);
        if (__syncthreads_or(!ok)) {
            // every group has left its loop: an update group whose copy did not land waits for it (bounded), so that
            // none is in flight into shared memory when the block exits (a copy is issued and awaited by the same
            // group, token by token)
            if (inflight >= 0)
                mbar_wait_bounded(slot_of(layer, g0 + inflight).bar, parity_of(layer, g0 + inflight));
            if (tid == 0) atomicOr(m.status, kStatusTimeout);
            return;
        }
        if (is_nll && gtid == 0) bits[s] = nll / 0.69314718055994530942;
        if (state != nullptr)
            for (int j = tid; j < L * N; j += nthr) {
                const int li = j / N, c = j % N;
                if (c < ns) state[((size_t)s * L + li) * ns + c] = qs[j];
            }
        g0 += T > 1 ? T - 1 : 0;
        __syncthreads();
    }
}

// ------------------------------------------------------------------------------------------------ launchers

template <int BLK, int R, int R2T, int LT, int NVT> static SmemLimits &coop_step_limit() { static SmemLimits l{}; return l; }
template <int BLK, int R, int R2T, int LT, int NVT> static SmemLimits &coop_score_limit() { static SmemLimits l{}; return l; }
template <int BLK, int R, int R2T, int LT, int NVT> static SmemLimits &pipe_score_limit() { static SmemLimits l{}; return l; }
template <int BLK, int R, int R2T, int LT, int NVT> static SmemLimits &split_score_limit() { static SmemLimits l{}; return l; }

template <int BLK, int R, int R2T, int LT, int NVT>
static cudaError_t coop_step_t(const DevModel &dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                               float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int sm_count,
                               cudaStream_t st) {
    const size_t smem = coop_smem_bytes(rec_max, 128, (dm.L * 128 + 127) / 128 * 128);
    cudaError_t e = raise_smem_limit((const void *)coop_step_kernel<BLK, R, R2T, LT, NVT>, smem,
                                     coop_step_limit<BLK, R, R2T, LT, NVT>());
    if (e != cudaSuccess) return e;
    const int grid = B < sm_count * kCoopBlocksPerSm ? B : sm_count * kCoopBlocksPerSm;
    coop_step_kernel<BLK, R, R2T, LT, NVT><<<grid, kCoopThreads, smem, st>>>(dm, B, tok, sin, sout, lg, routes, acc,
                                                                             rec_max);
    return cudaGetLastError();
}

template <int BLK, int R, int R2T, int LT, int NVT>
static cudaError_t coop_score_t(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                                uint32_t rec_max, int sm_count, cudaStream_t st) {
    const size_t smem = coop_smem_bytes(rec_max, 128, (dm.L * 128 + 127) / 128 * 128);
    cudaError_t e = raise_smem_limit((const void *)coop_score_kernel<BLK, R, R2T, LT, NVT>, smem,
                                     coop_score_limit<BLK, R, R2T, LT, NVT>());
    if (e != cudaSuccess) return e;
    const int grid = B < sm_count * kCoopBlocksPerSm ? B : sm_count * kCoopBlocksPerSm;
    coop_score_kernel<BLK, R, R2T, LT, NVT><<<grid, kCoopThreads, smem, st>>>(dm, B, T, tok, state, bits, rec_max);
    return cudaGetLastError();
}

template <int BLK, int R, int R2T, int LT, int NVT>
static cudaError_t pipe_score_t(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                                uint32_t rec_max, int sm_count, bool split, cudaStream_t st) {
    const int grid = B < sm_count ? B : sm_count;
    if (split && 2 * dm.L <= 8) {   // 2L groups of 128 threads: a router and an update group per routed layer
        const size_t smem = split_smem_bytes(rec_max, dm.L);
        cudaError_t e = raise_smem_limit((const void *)split_score_kernel<BLK, R, R2T, LT, NVT>, smem,
                                         split_score_limit<BLK, R, R2T, LT, NVT>());
        if (e != cudaSuccess) return e;
        split_score_kernel<BLK, R, R2T, LT, NVT><<<grid, 256 * dm.L, smem, st>>>(dm, B, T, tok, state, bits, rec_max);
        return cudaGetLastError();
    }
    if (dm.L + 1 > 8) return cudaErrorInvalidValue;   // L + 1 groups of 128 threads in one block
    const size_t smem = pipe_smem_bytes(rec_max, dm.L);
    cudaError_t e = raise_smem_limit((const void *)pipe_score_kernel<BLK, R, R2T, LT, NVT>, smem,
                                     pipe_score_limit<BLK, R, R2T, LT, NVT>());
    if (e != cudaSuccess) return e;
    pipe_score_kernel<BLK, R, R2T, LT, NVT><<<grid, 128 * (dm.L + 1), smem, st>>>(dm, B, T, tok, state, bits, rec_max);
    return cudaGetLastError();
}

// n = 128 only (the device layout's n; the d_state 96 extension included). Fast instances: c3 (V <= 32) and c4 / c5
// (V = 256); generic instances read R2, L and the classes at run time.
#define YGG_COOP_DISPATCH(FN, ...)                                                                            \
    if (dm.n != 128) return cudaErrorInvalidValue;                                                            \
    if (dm.b == 16 && dm.R == 16 && dm.R2P == 32 && dm.L == 4 && dm.VP == 32) return FN<16, 16, 32, 4, 1>(__VA_ARGS__); \
    if (dm.b == 16 && dm.R == 16 && dm.R2P == 32 && dm.L == 4 && dm.VP == 256) return FN<16, 16, 32, 4, 8>(__VA_ARGS__); \
    switch (dm.b * 100 + dm.R) {                                                                              \
        case 8 * 100 + 8: return FN<8, 8, 0, 0, 0>(__VA_ARGS__);                                              \
        case 8 * 100 + 16: return FN<8, 16, 0, 0, 0>(__VA_ARGS__);                                            \
        case 8 * 100 + 32: return FN<8, 32, 0, 0, 0>(__VA_ARGS__);                                            \
        case 16 * 100 + 8: return FN<16, 8, 0, 0, 0>(__VA_ARGS__);                                            \
        case 16 * 100 + 16: return FN<16, 16, 0, 0, 0>(__VA_ARGS__);                                          \
        case 16 * 100 + 32: return FN<16, 32, 0, 0, 0>(__VA_ARGS__);                                          \
        default: return cudaErrorInvalidValue;                                                                \
    }

cudaError_t launch_coop_step(const DevModel &dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                             float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int sm_count, cudaStream_t st) {
    YGG_COOP_DISPATCH(coop_step_t, dm, B, tok, sin, sout, lg, routes, acc, rec_max, sm_count, st)
}

cudaError_t launch_coop_score(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                              uint32_t rec_max, int sm_count, cudaStream_t st) {
    YGG_COOP_DISPATCH(coop_score_t, dm, B, T, tok, state, bits, rec_max, sm_count, st)
}

cudaError_t launch_pipe_score(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                              uint32_t rec_max, int sm_count, bool split, cudaStream_t st) {
    YGG_COOP_DISPATCH(pipe_score_t, dm, B, T, tok, state, bits, rec_max, sm_count, split, st)
}

}  // namespace ygg
