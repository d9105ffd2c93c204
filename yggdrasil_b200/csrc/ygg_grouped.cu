// Grouped scoring on sm_100a: rows of T tokens scored step by step and layer by layer. Per layer the streams are
// bucketed by the leaf they route to; a leaf that at least G streams share runs its expert update as int8 GEMMs on
// the 5th-generation tensor cores (tcgen05.mma kind::i8, accumulators in TMEM), the other streams take the per-stream
// path of the fused kernels. The results equal the fused score kernel bit for bit.
//
// One step is, for every layer l (the per-stream kernels serve a stream with G lanes, the model's lw: a warp, or half
// a warp with two streams per warp):
//   g_route    G lanes per stream: rho, router descent, layer-input codes; leaf id and its rank in the leaf's bucket
//   g_scan     one block: prefix sum of the per-leaf counts, the list of heavy leaves (count >= G) with the first of
//              their work items (one per tile of 128 of the leaf's streams), counts zeroed
//   g_scatter  thread per stream: heavy streams into their leaf's bucket, the others into the light list
//   g_heavy    the work items (leaf, tile) split into contiguous runs over the SMs' blocks, so that a hot leaf's
//              tiles run on many SMs; a block stages a leaf's weights into shared memory as K-major operands when its
//              run reaches the leaf, then per tile of 128 of its streams (M = streams, N = output features, K = input):
//                D_hi = Q_old . hi(A16)^T, D_lo = Q_old . lo(A16)^T          (A16 = 256 hi + lo, exact in int32)
//                D_u  = ZL . U'^T,  D_f = V(x) . U^T (factored input)
//              an epilogue per stream (thread = TMEM lane = stream) forms the int32 accumulators as the reference does,
//              saturates the new state into shared memory, and D_p = Q_new . P^T gives the readout codes
//   g_light    G lanes per stream on a light leaf: the per-stream update (leaf_update / readout_code)
// then g_head_nll: G lanes per stream, logits of all layers in order and the f64 NLL of the next token.
// A warp whose second stream is past the end runs a copy of its first unseen (nothing written), so that its
// collectives stay full-warp.
#include <cuda_runtime.h>
#include <stdint.h>

#include "ygg_device.cuh"

namespace ygg {

// Device workspace of the grouped path (caller-provided, carved by grouped_layout).
struct GroupWs {
    int32_t *leaf;      // [B] leaf of the current layer
    int32_t *pos;       // [B] rank of the stream in its leaf's bucket
    int32_t *member;    // [B] streams bucketed by leaf (heavy leaves only)
    int32_t *light;     // [B] streams on light leaves
    int32_t *cnt;       // [Emax] per-leaf counts (kept zero between layers)
    int32_t *off;       // [Emax + 1] bucket offsets
    int32_t *heavy;     // [Emax] heavy leaves
    int32_t *tile_off;  // [Emax + 1] first work item (128-stream tile) of each heavy leaf
    int32_t *counts;    // [3] heavy leaves, light streams, work items
    int8_t *zl;         // [B][64] layer-input codes
    int8_t *zq;         // [B][L][32] readout codes of every layer
    double *nll;        // [B]
    int8_t *state;      // [B][L][n] when the caller passes none
    int32_t *bad;       // [B] 1: the row holds a token outside [0, V); it is skipped and scores NaN
};

// Token t of row s, 0 for a row with a bad token (its results are discarded; this keeps every table index in range).
__device__ __forceinline__ int tok_at(const int32_t *tokens, const GroupWs &ws, int s, int T, int t) {
    return ws.bad[s] ? 0 : tokens[(size_t)s * T + t];
}

constexpr int kZlStride = 64;
constexpr int kZqStride = 32;
constexpr int kHeavyThreads = 128;

// ------------------------------------------------------------------------------------------------ tcgen05 helpers

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8 rows x 16 bytes, the K chunks of a row
// group 128 bytes apart (leading byte offset), row groups kbytes / 16 * 128 bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, int kbytes) {
    const uint64_t start = (saddr & 0x3FFFFu) >> 4;
    const uint64_t lbo = 128u >> 4;
    const uint64_t sbo = (uint64_t)(kbytes / 16 * 128) >> 4;
    return start | (lbo << 16) | (sbo << 32) | (1ull << 46);   // version 1, base offset 0, layout SWIZZLE_NONE
}
// Instruction descriptor of kind::i8: int32 accumulate, K-major A and B, M = 128, N = n_cols.
__device__ __forceinline__ uint32_t umma_idesc_i8(bool a_signed, bool b_signed, int n_cols) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(n_cols >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum ? 1u : 0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15},"
        " [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of (row, k) in a K-major no-swizzle operand with kbytes per row.
__device__ __forceinline__ int core_off(int row, int k, int kbytes) {
    return ((row >> 3) * (kbytes >> 4) + (k >> 4)) * 128 + (row & 7) * 16 + (k & 15);
}
// Row `row` of an operand: its kbytes bytes as kbytes / 16 chunks of 16 (chunk c of a row lands at one core matrix).
__device__ __forceinline__ void put_row16(uint8_t *op, int row, int kbytes, int chunk, const uint4 &v) {
    *(uint4 *)(op + core_off(row, 16 * chunk, kbytes)) = v;
}

__host__ __device__ constexpr int round32(int x) { return (x + 31) / 32 * 32; }

// Shared-memory plan of g_heavy for state width n, layer-input rank R2P, factored rank KP (0: table), readout rank R.
struct HeavyPlan {
    int ku, kf;                                      // K of the layer-input and factored GEMMs (multiples of 32)
    int o_hi, o_lo, o_u, o_f, o_p, o_aq, o_az, o_af, o_an, o_bar, bytes;
    __host__ __device__ HeavyPlan(int n, int r2p, int kp, int r) {
        ku = r2p ? round32(r2p) : 0;
        kf = kp ? round32(kp) : 0;
        int o = 0;
        auto take = [&](int b) { const int at = o; o += (b + 1023) / 1024 * 1024; return at; };
        o_hi = take(n * n);
        o_lo = take(n * n);
        o_u = take(n * ku);
        o_f = take(n * kf);
        o_p = take(r * n);
        o_aq = take(128 * n);
        o_az = take(128 * ku);
        o_af = take(128 * kf);
        o_an = take(128 * n);
        o_bar = take(256);
        bytes = o;
    }
};

// ------------------------------------------------------------------------------------------------ kernels

template <int N, int R2T, int G>
__global__ void __launch_bounds__(256) g_route(const __grid_constant__ DevModel m, int l, int B, int T, int t,
                                               const int32_t *__restrict__ tokens, const int8_t *state, GroupWs ws) {
    constexpr int C = N / G, P = 32 / G;
    __shared__ __align__(16) int8_t qb_s[8 * P][N];
    __shared__ __align__(16) int8_t zl_unseen[8 * P][kZlStride];   // where a stream that runs unseen writes
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gh = lane / G, gl = lane & (G - 1);
    const int base = (blockIdx.x * 8 + warp) * P;
    if (base >= B) return;
    const int s = base + gh;
    const bool real = s < B;
    const int se = real ? s : base;
    const int sidx = warp * P + gh;
    const int x = tok_at(tokens, ws, se, T, t);
    const DevLayer &y = m.layer[l];
    int leaf = x;
    if (l > 0) {
        const LaneQ<C> qbelow = load_q<C>(state + ((size_t)se * m.L + (l - 1)) * N + C * gl);
        const float rho = rms_rho<N, G>(qbelow, y.r2b, y.rms_eps, m.inv_n, lane);
        store_q<C>(qb_s[sidx] + C * gl, qbelow);
        __syncwarp();
        const uint4 qrow = *(const uint4 *)(qb_s[sidx] + 16 * (gl % (N / 16)));
        leaf = (m.D == 13 ? route_look<N, G, 13>(y.w, y.thr + (size_t)x * m.E, m.D, qrow, rho, lane)
                          : route_look<N, G>(y.w, y.thr + (size_t)x * m.E, m.D, qrow, rho, lane)) - m.E;
        if (R2T > 0 || m.R2 > 0)
            layer_input_codes<N, R2T, G>(m, y, qb_s[sidx], rho, real ? ws.zl + (size_t)s * kZlStride : zl_unseen[sidx],
                                         lane);
    }
    if (real && gl == 0) {
        ws.leaf[s] = leaf;
        ws.pos[s] = atomicAdd(ws.cnt + leaf, 1);
    }
}

// One block of 1024 threads: exclusive scan of cnt[0, n_leaves) into off, heavy leaves (count >= G) in leaf order with
// the first of their work items (tiles of 128 streams), counts zeroed for the next layer.
__global__ void __launch_bounds__(1024) g_scan(GroupWs ws, int n_leaves, int G) {
    __shared__ int part[1024];
    __shared__ int hpart[1024];
    __shared__ int tpart[1024];
    const int tid = threadIdx.x;
    const int per = (n_leaves + 1023) / 1024;
    const int a = min(tid * per, n_leaves), b = min(a + per, n_leaves);
    int sum = 0, hs = 0, ts = 0;
    for (int i = a; i < b; i++) {
        const int c = ws.cnt[i];
        sum += c;
        hs += c >= G;
        ts += c >= G ? (c + 127) / 128 : 0;
    }
    part[tid] = sum;
    hpart[tid] = hs;
    tpart[tid] = ts;
    __syncthreads();
    for (int d = 1; d < 1024; d <<= 1) {   // inclusive Hillis-Steele scan of the three arrays
        const int v = tid >= d ? part[tid - d] : 0, h = tid >= d ? hpart[tid - d] : 0, u = tid >= d ? tpart[tid - d] : 0;
        __syncthreads();
        part[tid] += v;
        hpart[tid] += h;
        tpart[tid] += u;
        __syncthreads();
    }
    int run = part[tid] - sum, hrun = hpart[tid] - hs, trun = tpart[tid] - ts;
    for (int i = a; i < b; i++) {
        const int c = ws.cnt[i];
        ws.off[i] = run;
        run += c;
        if (c >= G) {
            ws.tile_off[hrun] = trun;
            trun += (c + 127) / 128;
            ws.heavy[hrun++] = i;
        }
        ws.cnt[i] = 0;
    }
    if (tid == 1023) {
        ws.off[n_leaves] = part[1023];
        ws.counts[0] = hpart[1023];
        ws.counts[1] = 0;
        ws.counts[2] = tpart[1023];
        ws.tile_off[hpart[1023]] = tpart[1023];
    }
}

__global__ void g_scatter(GroupWs ws, int B, int G) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= B) return;
    const int leaf = ws.leaf[s];
    const int o = ws.off[leaf];
    if (ws.off[leaf + 1] - o >= G) ws.member[o + ws.pos[s]] = s;
    else ws.light[atomicAdd(ws.counts + 1, 1)] = s;
}

template <int N, int BLK, int R, int R2T, int G>
__global__ void __launch_bounds__(256) g_light(const __grid_constant__ DevModel m, int l, int T, int t,
                                               const int32_t *__restrict__ tokens, int8_t *state, GroupWs ws) {
    constexpr int C = N / G, P = 32 / G;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5, gh = lane / G,
              gl = lane & (G - 1);
    const int nlight = ws.counts[1];
    const DevLayer &y = m.layer[l];
    const bool low = l > 0 && (R2T > 0 || m.R2 > 0);
    for (int base = (blockIdx.x * W + warp) * P; base < nlight; base += gridDim.x * W * P) {
        const bool real = base + gh < nlight;
        const int s = ws.light[real ? base + gh : base];
        const int x = tok_at(tokens, ws, s, T, t);
        const int r = ws.leaf[s];
        const uint8_t *rec = y.rec + (size_t)r * y.rec_bytes;
        const int16_t *trow =
            y.table ? y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N : nullptr;
        int8_t *q = state + ((size_t)s * m.L + l) * N;
        int acc[C];
        LaneQ<C> qn;
        leaf_update<N, BLK, R2T, G>(m, y, rec, trow, x, q, ws.zl + (size_t)s * kZlStride, low, lane, acc, qn);
        __syncwarp();                              // every lane has read the old state before it is overwritten
        if (real) store_q<C>(q + C * gl, qn);
        const ReadoutPart<N, R, G> ro = readout_partials<N, R, G>(y, rec, qn, lane);
        const int zq = readout_code<N, R, G>(ro, lane);
        const int row = readout_row<R, G>(gl);
        if (real && row >= 0 && (G == 32 || R == 16 || (gl & 1) == 0))
            ws.zq[((size_t)s * m.L + l) * kZqStride + row] = (int8_t)zq;
    }
}

// Work items (heavy leaf, tile of up to 128 of its streams) in contiguous runs per block, 128 threads; a block stages a
// leaf's weights when its run reaches the leaf (a hot leaf's tiles spread over many blocks). Thread i is TMEM lane i:
// stream i of the tile in the epilogue, output row i of the leaf when the weights are staged.
template <int N, int BLK, int R, int R2T, int G>
__global__ void __launch_bounds__(kHeavyThreads, 1) g_heavy(const __grid_constant__ DevModel m, int l, int T, int t,
                                                             const int32_t *__restrict__ tokens, int8_t *state,
                                                             GroupWs ws) {
    constexpr int C = N / G;                   // the record layout: coordinates per lane, interleaved over G lanes
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5;
    const DevLayer &y = m.layer[l];
    const bool low = l > 0 && (R2T > 0 || m.R2 > 0);
    const bool fact = y.table == nullptr;
    const int R2P = R2T ? R2T : m.R2P, KP = m.KP;
    const HeavyPlan hp(N, low ? R2P : 0, fact ? KP : 0, R);
    uint8_t *bhi = smem + hp.o_hi, *blo = smem + hp.o_lo, *bu = smem + hp.o_u, *bf = smem + hp.o_f,
            *bp = smem + hp.o_p, *aq = smem + hp.o_aq, *az = smem + hp.o_az, *af = smem + hp.o_af,
            *an = smem + hp.o_an;
    uint32_t *tmem_slot = (uint32_t *)(smem + hp.o_bar + 16);
    float *mzs = (float *)(smem + hp.o_bar + 32);           // the leaf's per-row readout scales
    const uint32_t bar = smem_addr(smem + hp.o_bar);
    const int nheavy = ws.counts[0], nitems = ws.counts[2];
    const int per = (nitems + (int)gridDim.x - 1) / (int)gridDim.x;
    const int it0 = (int)blockIdx.x * per, it1 = min(it0 + per, nitems);
    if (it0 >= it1) return;

    // TMEM: D_hi [0, N), D_lo [N, 2N), D_u [2N, 3N), D_f [3N, 4N); the readout D_p reuses [0, R)
    constexpr uint32_t kCols = N <= 64 ? 256 : 512;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    uint32_t phase = 0;
    bool ok = true;
    const int rnd = 1 << (m.shift - 1), sh = m.shift;
    const uint32_t id_ss_n = umma_idesc_i8(true, true, N), id_su_n = umma_idesc_i8(true, false, N);
    const uint32_t id_ss_r = umma_idesc_i8(true, true, R);
    const int lane_base = (warp * 32) << 16;

    int staged = -1;   // the heavy leaf whose weights are in shared memory
    for (int it = it0; it < it1 && ok; it++) {
        // the item's heavy leaf: the last h with tile_off[h] <= it
        int lo = 0, hi = nheavy - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (ws.tile_off[mid] <= it) lo = mid; else hi = mid - 1;
        }
        const int h = lo, base = 128 * (it - ws.tile_off[h]);
        const int r = ws.heavy[h];
        const uint8_t *rec = y.rec + (size_t)r * y.rec_bytes;
        const int first = ws.off[r], count = ws.off[r + 1] - first;
        // ---- the leaf's weights as K-major B operands (row = output feature), once per run of its tiles
        if (h != staged) {
            staged = h;
            if (tid < N) {
                const int i = tid, ln = i / C, ii = i % C, c0 = (i / BLK) * BLK;
                for (int c = 0; c < N / 16; c++) {
                    put_row16(bhi, i, N, c, make_uint4(0, 0, 0, 0));
                    put_row16(blo, i, N, c, make_uint4(0, 0, 0, 0));
                }
                const uint8_t *pa = rec + y.off_a;
                for (int p = 0; p < BLK / 2; p++) {
                    const int lb = (ii * (BLK / 2) + p) * 4;                   // the lane's byte of the int16 pair
                    const uint32_t wv = *(const uint32_t *)(pa + ((lb / 16) * G + ln) * 16 + lb % 16);
                    const int a0 = (int)(int16_t)(wv & 0xFFFFu), a1 = (int)(int16_t)(wv >> 16);
                    bhi[core_off(i, c0 + 2 * p, N)] = (uint8_t)(a0 >> 8);
                    blo[core_off(i, c0 + 2 * p, N)] = (uint8_t)(a0 & 0xFF);
                    bhi[core_off(i, c0 + 2 * p + 1, N)] = (uint8_t)(a1 >> 8);
                    blo[core_off(i, c0 + 2 * p + 1, N)] = (uint8_t)(a1 & 0xFF);
                }
                if (low) {
                    const uint8_t *pu = rec + y.off_u;
                    for (int k = 0; k < hp.ku; k++) {
                        const int lb = ii * R2P + k;
                        bu[core_off(i, k, hp.ku)] = k < R2P ? pu[((lb / 16) * G + ln) * 16 + lb % 16] : 0;
                    }
                }
                if (fact) {
                    const uint8_t *pf = rec + y.off_f;
                    for (int k = 0; k < hp.kf; k++) {
                        const int lb = ii * KP + k;
                        bf[core_off(i, k, hp.kf)] = k < KP ? pf[((lb / 16) * G + ln) * 16 + lb % 16] : 0;
                    }
                }
            }
            if (tid < R) {
                const uint8_t *pp = rec + y.off_p;
                for (int i = 0; i < N; i++) {
                    const int lb = tid * C + i % C, ln = i / C;
                    bp[core_off(tid, i, N)] = pp[((lb / 16) * G + ln) * 16 + lb % 16];
                }
            }
            if (tid < R) mzs[tid] = y.off_mz != kNone ? *(const float *)(rec + y.off_mz + 4 * tid) : y.readout_scale;
        }
        const float su = fact ? *(const float *)(rec + y.off_su) : 0.0f;
        // ---- the item's tile of up to 128 streams
        {
            const int ntile = min(128, count - base);
            const int s = tid < ntile ? ws.member[first + base + tid] : -1;
            const int x = s >= 0 ? tok_at(tokens, ws, s, T, t) : 0;
            int8_t *qrow = s >= 0 ? state + ((size_t)s * m.L + l) * N : nullptr;
            for (int c = 0; c < N / 16; c++)
                put_row16(aq, tid, N, c, s >= 0 ? *(const uint4 *)(qrow + 16 * c) : make_uint4(0, 0, 0, 0));
            if (low)
                for (int c = 0; c < hp.ku / 16; c++)
                    put_row16(az, tid, hp.ku, c,
                              (s >= 0 && 16 * c < R2P) ? *(const uint4 *)(ws.zl + (size_t)s * kZlStride + 16 * c)
                                                       : make_uint4(0, 0, 0, 0));
            if (fact)
                for (int c = 0; c < hp.kf / 16; c++)
                    put_row16(af, tid, hp.kf, c,
                              (s >= 0 && 16 * c < KP) ? __ldg((const uint4 *)(y.vt + (size_t)x * KP + 16 * c))
                                                      : make_uint4(0, 0, 0, 0));
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                const uint32_t saq = smem_addr(aq);
                for (int ks = 0; ks < N / 32; ks++) {
                    const uint64_t ad = umma_desc(saq + ks * 256, N);
                    umma_i8(tmem + 0, ad, umma_desc(smem_addr(bhi) + ks * 256, N), id_ss_n, ks > 0);
                    umma_i8(tmem + N, ad, umma_desc(smem_addr(blo) + ks * 256, N), id_su_n, ks > 0);
                }
                if (low)
                    for (int ks = 0; ks < hp.ku / 32; ks++)
                        umma_i8(tmem + 2 * N, umma_desc(smem_addr(az) + ks * 256, hp.ku),
                                umma_desc(smem_addr(bu) + ks * 256, hp.ku), id_ss_n, ks > 0);
                if (fact)
                    for (int ks = 0; ks < hp.kf / 32; ks++)
                        umma_i8(tmem + 3 * N, umma_desc(smem_addr(af) + ks * 256, hp.kf),
                                umma_desc(smem_addr(bf) + ks * 256, hp.kf), id_ss_n, ks > 0);
                umma_commit(bar);
            }
            ok = mbar_wait_bounded(bar, phase);
            phase ^= 1u;
            ok = __syncthreads_and(ok);
            if (!ok) break;
            tc_fence_after();
            // ---- epilogue: thread tid owns stream row tid; columns in chunks of 16
            const int16_t *trow =
                (s >= 0 && !fact) ? y.table + ((size_t)r * y.table_rows + (y.table_rows > 1 ? x : 0)) * N : nullptr;
            for (int c0 = 0; c0 < N; c0 += 16) {
                uint32_t vh[16], vl[16], vu[16], vf[16];
                tmem_ld16(tmem + lane_base + c0, vh);
                tmem_ld16(tmem + lane_base + N + c0, vl);
                if (low) tmem_ld16(tmem + lane_base + 2 * N + c0, vu);
                if (fact) tmem_ld16(tmem + lane_base + 3 * N + c0, vf);
                tmem_ld_wait();
                uint32_t packed[4] = {0, 0, 0, 0};
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int i = c0 + j;
                    int acc = ((int)vh[j] * 256 + (int)vl[j] + rnd) >> sh;
                    if (s >= 0) {
                        if (fact) {
                            const float mul = __fmul_rn(su, __ldg(y.mt + i));
                            acc += cvt_rne(__fmul_rn(i2f((int)vf[j]), mul)) + *(const int16_t *)(rec + y.off_cb + 2 * i);
                        } else {
                            acc += trow[i];
                        }
                        if (low) {
                            const float mu = y.mulv ? __ldg(y.mulv + i) : y.layer_input_scale;
                            acc += cvt_rne(__fmul_rn(i2f((int)vu[j]), mu));
                        }
                    }
                    packed[j >> 2] |= (uint32_t)(uint8_t)(int8_t)clampi(acc, -128, 127) << (8 * (j & 3));
                }
                const uint4 v = s >= 0 ? make_uint4(packed[0], packed[1], packed[2], packed[3]) : make_uint4(0, 0, 0, 0);
                put_row16(an, tid, N, c0 / 16, v);
                if (s >= 0) *(uint4 *)(qrow + c0) = v;
            }
            // ---- readout D_p = Q_new . P^T into columns [0, R)
            fence_proxy_async();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
                for (int ks = 0; ks < N / 32; ks++)
                    umma_i8(tmem + 0, umma_desc(smem_addr(an) + ks * 256, N), umma_desc(smem_addr(bp) + ks * 256, N),
                            id_ss_r, ks > 0);
                umma_commit(bar);
            }
            ok = mbar_wait_bounded(bar, phase);
            phase ^= 1u;
            ok = __syncthreads_and(ok);
            if (!ok) break;
            tc_fence_after();
            for (int c0 = 0; c0 < R; c0 += 16) {
                uint32_t vz[16];
                if (R >= 16 || c0 == 0) tmem_ld16(tmem + lane_base + c0, vz);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int rr = c0 + j;
                    if (rr < R && s >= 0)
                        ws.zq[((size_t)s * m.L + l) * kZqStride + rr] =
                            (int8_t)clampi(cvt_rne(__fmul_rn(i2f((int)vz[j]), mzs[rr])), -127, 127);
                }
            }
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
        }
    }
    if (!ok && tid == 0) atomicOr(m.status, kStatusTimeout);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
}

template <int R, int NVT, int G>
__global__ void __launch_bounds__(256) g_head_nll(const __grid_constant__ DevModel m, int B, int T, int t,
                                                  const int32_t *__restrict__ tokens, GroupWs ws, double *bits) {
    constexpr int P = 32 / G;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gh = lane / G, gl = lane & (G - 1);
    const int base = (blockIdx.x * 8 + warp) * P;
    if (base >= B) return;
    const int s = base + gh < B ? base + gh : base;
    const bool live = base + gh < B && !ws.bad[s];
    const int nv = NVT ? NVT : m.VP / G;
    float lg[kMaxClasses<G>];
#pragma unroll
    for (int c = 0; c < kMaxClasses<G>; c++) lg[c] = c < nv ? __ldg(m.head_b + G * c + gl) : 0.0f;
    for (int l = 0; l < m.L; l++)
        head_accumulate<R, NVT, G>(m, m.layer[l], ws.zq + ((size_t)s * m.L + l) * kZqStride, lg, lane);
    const double nll = ws.nll[s] + nll_of<G>(lg, nv, m.V, live ? tokens[(size_t)s * T + t + 1] : 0, lane);
    if (live && gl == 0) {
        ws.nll[s] = nll;
        if (t + 2 == T) bits[s] = nll / 0.69314718055994530942;
    }
}

// Rows with a token out of range are skipped and score NaN, as in the fused score kernel (cpu/ygg.cpp:493-495
// rejects the whole input); the status word records it.
__global__ void g_check(int B, int T, int V, const int32_t *__restrict__ tokens, int *status, double *bits,
                        int32_t *bad) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= B) return;
    int b = 0;
    for (int t = 0; t < T; t++) b |= tokens[(size_t)s * T + t] < 0 || tokens[(size_t)s * T + t] >= V;
    bad[s] = b;
    if (b) {
        atomicOr(status, kStatusBadToken);
        bits[s] = __longlong_as_double(0x7ff8000000000000LL);
    }
}

// The caller's state [B][L][ns] to and from the device layout [B][L][N] of a model whose n is padded (ns < N): the
// grouped kernels then work on the padded copy, whose extra coordinates start and stay 0.
__global__ void g_state_pad(int B, int L, int ns, int N, const int8_t *__restrict__ src, int8_t *__restrict__ dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)B * L * N) return;
    const size_t row = i / N;
    const int c = (int)(i % N);
    dst[i] = (src != nullptr && c < ns) ? src[row * ns + c] : (int8_t)0;
}
__global__ void g_state_unpad(int B, int L, int ns, int N, const int8_t *__restrict__ src, int8_t *__restrict__ dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)B * L * ns) return;
    dst[i] = src[(i / ns) * N + i % ns];
}

// ------------------------------------------------------------------------------------------------ host side

size_t grouped_ws_bytes(const DevModel &m, int B) {
    const size_t Emax = (size_t)(m.E > m.V ? m.E : m.V);
    auto r = [](size_t x) { return (x + 255) / 256 * 256; };
    return r(4 * (size_t)B) * 5 + r(4 * Emax) * 2 + r(4 * (Emax + 1)) * 2 + 256 + r((size_t)B * kZlStride) +
           r((size_t)B * m.L * kZqStride) + r(8 * (size_t)B) + r((size_t)B * m.L * m.n);
}

static GroupWs grouped_layout(const DevModel &m, int B, uint8_t *base) {
    const size_t Emax = (size_t)(m.E > m.V ? m.E : m.V);
    auto r = [](size_t x) { return (x + 255) / 256 * 256; };
    size_t o = 0;
    auto take = [&](size_t b) { uint8_t *p = base + o; o += r(b); return p; };
    GroupWs ws;
    ws.leaf = (int32_t *)take(4 * (size_t)B);
    ws.pos = (int32_t *)take(4 * (size_t)B);
    ws.member = (int32_t *)take(4 * (size_t)B);
    ws.light = (int32_t *)take(4 * (size_t)B);
    ws.bad = (int32_t *)take(4 * (size_t)B);
    ws.cnt = (int32_t *)take(4 * Emax);
    ws.heavy = (int32_t *)take(4 * Emax);
    ws.tile_off = (int32_t *)take(4 * (Emax + 1));
    ws.off = (int32_t *)take(4 * (Emax + 1));
    ws.counts = (int32_t *)take(256);
    ws.zl = (int8_t *)take((size_t)B * kZlStride);
    ws.zq = (int8_t *)take((size_t)B * m.L * kZqStride);
    ws.nll = (double *)take(8 * (size_t)B);
    ws.state = (int8_t *)take((size_t)B * m.L * m.n);
    return ws;
}

// LG: lanes per stream of the per-stream kernels (the model's lw); G: streams a leaf needs for the tensor-core path.
template <int N, int BLK, int R, int R2T, int NVT, int LG>
static cudaError_t run_grouped_t(const DevModel &m, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                                 void *workspace, int G, int sm_count, cudaStream_t st) {
    GroupWs ws = grouped_layout(m, B, (uint8_t *)workspace);
    // the caller's state in place, unless there is none (zero start) or its layout is narrower than the device's
    const bool padded = m.ns != N;
    int8_t *q = (state && !padded) ? state : ws.state;
    const size_t Emax = (size_t)(m.E > m.V ? m.E : m.V);
    cudaError_t e = cudaMemsetAsync(ws.cnt, 0, 4 * Emax, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ws.nll, 0, 8 * (size_t)B, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(bits, 0, 8 * (size_t)B, st);
    if (e == cudaSuccess && !state && !padded) e = cudaMemsetAsync(ws.state, 0, (size_t)B * m.L * N, st);
    if (e != cudaSuccess) return e;
    const size_t cells = (size_t)B * m.L * N;
    if (padded) g_state_pad<<<(unsigned)((cells + 255) / 256), 256, 0, st>>>(B, m.L, m.ns, N, state, ws.state);
    g_check<<<(B + 255) / 256, 256, 0, st>>>(B, T, m.V, tok, m.status, bits, ws.bad);
    if (T < 2) return cudaGetLastError();   // no next token to score
    // N = 256 has no tensor-core path (its operands do not fit a block's shared memory): every stream is light
    constexpr bool tc = N <= 128;
    const int Geff = tc ? (G < 1 ? 1 : G) : (1 << 30);
    const HeavyPlan hp(N, m.R2P, m.factored ? m.KP : 0, R);
    if constexpr (tc) {
        static SmemLimits lim{};
        e = raise_smem_limit((const void *)g_heavy<N, BLK, R, R2T, LG>, (size_t)hp.bytes, lim);
        if (e != cudaSuccess) return e;
    }
    constexpr int P = 32 / LG;   // streams per warp
    const int rb = (B + 8 * P - 1) / (8 * P);
    const int lb = rb < 4 * sm_count ? rb : 4 * sm_count;
    for (int t = 0; t + 1 < T; t++) {
        for (int l = 0; l < m.L; l++) {
            const int n_leaves = l == 0 ? m.V : m.E;
            g_route<N, R2T, LG><<<rb, 256, 0, st>>>(m, l, B, T, t, tok, q, ws);
            g_scan<<<1, 1024, 0, st>>>(ws, n_leaves, Geff);
            g_scatter<<<(B + 255) / 256, 256, 0, st>>>(ws, B, Geff);
            if constexpr (tc)
                g_heavy<N, BLK, R, R2T, LG><<<sm_count, kHeavyThreads, hp.bytes, st>>>(m, l, T, t, tok, q, ws);
            g_light<N, BLK, R, R2T, LG><<<lb, 256, 0, st>>>(m, l, T, t, tok, q, ws);
        }
        g_head_nll<R, NVT, LG><<<rb, 256, 0, st>>>(m, B, T, t, tok, ws, bits);
    }
    if (padded && state)
        g_state_unpad<<<(unsigned)(((size_t)B * m.L * m.ns + 255) / 256), 256, 0, st>>>(B, m.L, m.ns, N, ws.state, state);
    return cudaGetLastError();
}

cudaError_t run_grouped(int n, int blk, int r, int r2p, const DevModel &m, int B, int T, const int32_t *tok,
                        int8_t *state, double *bits, void *workspace, int G, int sm_count, cudaStream_t st) {
    const int VP = m.VP;
    if (m.lw == 16) {
        if (n == 128 && blk == 16 && r == 16 && r2p == 32 && VP == 32)
            return run_grouped_t<128, 16, 16, 32, 2, 16>(m, B, T, tok, state, bits, workspace, G, sm_count, st);
        if (n == 128 && blk == 16 && r == 16 && r2p == 32 && VP == 256)
            return run_grouped_t<128, 16, 16, 32, 16, 16>(m, B, T, tok, state, bits, workspace, G, sm_count, st);
        switch (n * 1000 + blk * 100 + r) {
#define YGG_G(N_, B_, R_) \
    case N_ * 1000 + B_ * 100 + R_: return run_grouped_t<N_, B_, R_, 0, 0, 16>(m, B, T, tok, state, bits, workspace, G, sm_count, st);
            YGG_G(64, 8, 8) YGG_G(64, 8, 16) YGG_G(64, 16, 8) YGG_G(64, 16, 16)
            YGG_G(128, 8, 8) YGG_G(128, 8, 16) YGG_G(128, 16, 8) YGG_G(128, 16, 16)
#undef YGG_G
            default: return cudaErrorInvalidValue;
        }
    }
    if (n == 128 && blk == 16 && r == 16 && r2p == 32 && VP == 32)
        return run_grouped_t<128, 16, 16, 32, 1, 32>(m, B, T, tok, state, bits, workspace, G, sm_count, st);
    if (n == 128 && blk == 16 && r == 16 && r2p == 32 && VP == 256)
        return run_grouped_t<128, 16, 16, 32, 8, 32>(m, B, T, tok, state, bits, workspace, G, sm_count, st);
    switch (n * 1000 + blk * 100 + r) {
#define YGG_G(N_, B_, R_) \
    case N_ * 1000 + B_ * 100 + R_: return run_grouped_t<N_, B_, R_, 0, 0, 32>(m, B, T, tok, state, bits, workspace, G, sm_count, st);
        YGG_G(64, 8, 8) YGG_G(64, 8, 16) YGG_G(64, 8, 32) YGG_G(64, 16, 8) YGG_G(64, 16, 16) YGG_G(64, 16, 32)
        YGG_G(128, 8, 8) YGG_G(128, 8, 16) YGG_G(128, 8, 32) YGG_G(128, 16, 8) YGG_G(128, 16, 16) YGG_G(128, 16, 32)
        YGG_G(256, 8, 8) YGG_G(256, 8, 16) YGG_G(256, 8, 32) YGG_G(256, 16, 8) YGG_G(256, 16, 16) YGG_G(256, 16, 32)
#undef YGG_G
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace ygg

// ------------------------------------------------------------------------------------------------ fixed scratch
//
// Scratch for callers that cannot allocate device memory while they run: a host that has handed every byte of the
// GPU to its own pool, a real-time serving loop that forbids allocation on its hot path, or a foreign-language
// binding with no CUDA allocator of its own. ygg_score_grouped_noalloc uses this array instead of a caller
// workspace. It is a fixed, modest size (kNoAllocScratchBytes), and every GPU that loads this library holds it until
// the process exits. All calls share it and it keeps the last call's contents, so each call clears what must start
// at zero, and calls whose work overlaps on the GPU (several streams, several host threads) race on it.
#include <mutex>

namespace ygg {
constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;   // 16 MiB
}

static __device__ __align__(256) uint8_t g_noalloc_scratch[ygg::kNoAllocScratchBytes];

namespace ygg {

// The context current on this thread (the driver's cuCtxGetCurrent, reached through the runtime's entry-point query
// so that the library needs no link against the driver library); null when it cannot be asked.
static void *current_context() {
    using CtxGetCurrent = int (*)(void **);
    static CtxGetCurrent fn = [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (CtxGetCurrent) nullptr;
        return (CtxGetCurrent)f;
    }();
    void *ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != 0) return nullptr;
    return ctx;
}

// The device address of the fixed scratch on `device`, which must be the current device. The array's name is only a
// host-side handle, so the address is looked up (cudaGetSymbolAddress) the first time a device is seen and cached
// with the context it belongs to; when the device's context is another one by the next call (the primary context
// was reset, or a different context was made current), the address is looked up again.
cudaError_t noalloc_scratch(int device, void **ptr, size_t *bytes) {
    constexpr int kMaxDev = 64;
    static std::mutex mu;
    static void *addr[kMaxDev] = {};
    static void *owner[kMaxDev] = {};
    if (device < 0 || device >= kMaxDev) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    void *ctx = current_context();
    if (addr[device] == nullptr || ctx == nullptr || ctx != owner[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        addr[device] = p;
        owner[device] = current_context();   // the lookup above made the device's context current if it was not
    }
    *ptr = addr[device];
    *bytes = kNoAllocScratchBytes;
    return cudaSuccess;
}

}  // namespace ygg
