// The fp32 streaming step of Yggdrasil on sm_100a: the reference's float inference model (yggdrasil/inference.py:42-75;
// its Triton backend fuses the same step, yggdrasil/inference_triton.py:21-106, and adds the head with torch.addmm,
// :187-194), as the backend "b200f".
//
// One block serves one stream at a time (grid-stride over the streams): n threads, thread t owning state coordinate t
// of every layer, for large batches; 4 n threads for a batch of at most two streams per SM, where a step's time is
// its chain of dependent loads: four quarter-blocks, quarter s taking the terms s mod 4 of every coordinate's sums
// (a warp then holds 32 consecutive coordinates, so its expert loads are whole lines). Per layer:
//   1. the router (routed layers): f = [router_embed(x); rms(h_below)], node j goes right iff f . W_j + b_j > 0,
//      descended kLook = 4 levels per round: the 15 rows of the subtree under the current node are loaded together
//      (every load issued before any is used, so a round costs one memory latency), thread t multiplying feature t of
//      each row, and one reduction of the 15 partial sums decides the round (inference.py:42-52). At small batches
//      only the warps that hold a feature route, reading a copy of the rows blocked by round (a thread's weights
//      are four 16-byte loads), with one named barrier per round;
//   2. the layer input v = V' rms(h_below) (the inputs split over the threads, then the parts added; at small batches
//      V' is copied into shared memory while the layer below finishes and summed by the warps that do not route,
//      while the others route), an L2 prefetch of the chosen expert's arrays, then h_t = T_r[x][t] + sum_k U'_r[t][k]
//      v_k + sum_j A_r[t][j] h_prev[block(t) + j] (inference.py:55-63); every expert array is stored transposed so
//      that each of these loads is coalesced over the block's threads;
//   3. the readout z = P_r h (a reduce-scatter within each warp, then the warps' sums added; at small batches per
//      quarter-block, with the sum of h^2, behind two barriers) and rms(h) for the layer above.
// At small batches, helper blocks past the streams' prefetch the arrays every stream reads (router rows, V', Q) into
// L2 at the start of the launch, and a stream's state and router embeddings of every layer are read at once.
// The logits are output_bias + sum_l z_l Q_l^T: at small batches added at each layer's readout, else after the last
// layer, one class per thread. Everything is fp32 with fused multiply-adds; the reference's own fp32 sums run in
// other orders, so parity is a tolerance (the reference's own: log-probabilities within 1e-4,
// cpu/tests/test_triton.py:29-30).
#include <algorithm>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "../../include/ygg_b200.h"

namespace ygg {
namespace fstep {

constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr int kMaxLayers = 16;
constexpr int kLook = 4;                       // router levels per round
constexpr int kVtSmem = 16384;                 // floats: V' (n x R2) is staged in shared memory up to this size
constexpr float kRmsEps = 1e-6f;               // yggdrasil/config.py:8

struct FLayer {
    const float *table;   // token layer [V][n] (T_x[x]); routed [E][V][n]
    const float *at;      // [E][b][n]: at[e][j][i] = A_e[i][block(i) b + j]; null: no transition
    const float *pt;      // readout [E][R][n]
    const float *qt;      // unembedding, transposed [R][C]
    const float *embed;   // router_embed [V][F] (routed layers)
    const float *w;       // router rows [E - 1][FIN], heap order from node 0
    const float *bias;    // [E - 1]
    const float *wb;      // the router rows again, blocked by round for the small-batch step: for each round (kLook
                          // levels from depth d0 = kLook i), for each node m of depth d0 in order, a block of the
                          // P - 1 rows of the subtree under m (P = 2^levels of the round) in local heap order (row k =
                          // 0 the node itself), stored [P/4][FIN][4]: element (k, f) at ((k/4) FIN + f) 4 + k mod 4,
                          // so that feature f's four rows 4q..4q+3 are one 16-byte load and a warp's loads coalesce
                          // ([FIN][2] for P = 2); row P - 1 is zero
    const float *vt;      // layer-input down projection, transposed [n][R2]; null: no layer input
    const float *ut;      // layer-input projection [E][R2][n]
};

struct FModel {
    int L, n, b, V, C, D, F, FIN, R, R2;
    int route_on_state;
    const float *out_bias;   // [C]
    FLayer layer[kMaxLayers];
};

template <int K> struct Log2 { static constexpr int value = K <= 1 ? 0 : 1 + Log2<K / 2>::value; };
template <> struct Log2<1> { static constexpr int value = 0; };

// Warp reduce-scatter of K values (K a power of two <= 32): halving exchanges from offset 16 down leave lane l with the
// warp sum of v[l >> (5 - log2 K)], then plain butterflies over the lower offsets.
template <int K> __device__ __forceinline__ float reduce_scatter(float (&v)[K], int lane) {
    constexpr int LK = Log2<K>::value;
#pragma unroll
    for (int s = 0; s < LK; s++) {
        const int off = 16 >> s;
        const int half = K >> (s + 1);
        const bool hi = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; i++) {
            const float keep = hi ? v[i + half] : v[i], send = hi ? v[i] : v[i + half];
            v[i] = keep + __shfl_xor_sync(kFull, send, off);
        }
    }
    float r = v[0];
#pragma unroll
    for (int off = 16 >> LK; off > 0; off >>= 1) r += __shfl_xor_sync(kFull, r, off);
    return r;
}

// Block sums of K per-thread values into out[0, K) (shared memory); red: NW * K floats of shared scratch. Each warp
// reduce-scatters its K sums into red, then a group of NW lanes per value adds the warps' sums with shuffles. Ends
// synchronised, so out[] is visible to every thread. Needs K <= 32 (K NW <= the block's threads).
template <int K, int NW>
__device__ __forceinline__ void block_sum(float (&v)[K], float *red, float *out, int tid) {
    constexpr int LK = Log2<K>::value;
    const int lane = tid & 31, warp = tid >> 5;
    const float r = reduce_scatter<K>(v, lane);
    if ((lane & ((32 >> LK) - 1)) == 0) red[warp * K + (lane >> (5 - LK))] = r;
    __syncthreads();
    constexpr int kActive = K * NW, kLanes = (kActive + 31) / 32 * 32;   // whole warps take part in the shuffles
    if (tid < kLanes) {
        float a = tid < kActive ? red[(tid % NW) * K + tid / NW] : 0.0f;
#pragma unroll
        for (int off = NW / 2; off > 0; off >>= 1) a += __shfl_xor_sync(kFull, a, off);
        if (tid < kActive && tid % NW == 0) out[tid / NW] = a;
    }
    __syncthreads();
}

// Bulk prefetch of `bytes` (16-aligned, a multiple of 16) of global memory into L2; nothing waits for it.
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 prefetch of `count` floats from p (256-byte aligned) in 16 KB pieces, piece i issued by thread i mod nthreads
// (g: this thread's index among them)
__device__ __forceinline__ void prefetch_spread(const float *p, size_t count, unsigned g, unsigned nthreads) {
    constexpr size_t kPiece = 4096;   // floats
    const size_t pieces = (count + kPiece - 1) / kPiece;
    for (size_t i = g; i < pieces; i += nthreads) {
        const size_t n = min(kPiece, count - i * kPiece) & ~size_t(3);
        if (n) prefetch_l2(p + i * kPiece, (uint32_t)(n * 4));
    }
}

// Barrier `id` (not 0, which __syncthreads uses) among the first `count` threads (a multiple of 32) of the block
__device__ __forceinline__ void named_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// One-thread bulk copy of `bytes` (16-byte aligned, a multiple of 16) global -> this block's shared memory, completing
// on the mbarrier at `bar` (which expects the bytes); and a bounded wait for a phase of that mbarrier (false: the
// copy did not land within the limit)
__device__ __forceinline__ void bulk_to_shared(float *dst, const float *src, uint32_t bytes, uint64_t *bar) {
    const unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src), "r"(bytes), "r"(b) : "memory");
}
__device__ __forceinline__ bool wait_phase(uint64_t *bar, unsigned parity) {
    const unsigned b = (unsigned)__cvta_generic_to_shared(bar);
    for (int i = 0; i < (1 << 22); i++) {   // each try may suspend the thread for a while: seconds in all
        unsigned ok;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(ok) : "r"(b), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}

// atomicMax of a non-negative float through its bits (the order of non-negative floats is that of their bits)
__device__ __forceinline__ void max_into(unsigned *p, float v) { atomicMax(p, __float_as_uint(fabsf(v))); }

// One stream per block of N * TPR threads at a time: thread t works on state coordinate t / TPR and takes part t % TPR
// of that coordinate's sums (TPR = 1 for throughput at large batches, 4 for the latency of small ones). state
// [B][L][n] (in may equal out), logits [B][C], experts [B][L] or null. RP: the readout rank rounded up to a power of
// two (<= 32). stats: null, or the calibration maxima of cpu/export.py:129-153 accumulated over the launch's streams,
// per layer [n/16 group maxima of |h|][max |V' rms(h_below)|][R row maxima of |P_r h|] as float bits (the caller
// zeroes them; an atomicMax per value and warp).
template <int N, int RP, int TPR>
__global__ void __launch_bounds__(N * TPR, TPR == 1 ? 1024 / N : 1) fstep_kernel(const __grid_constant__ FModel m, int B,
                                                        const int32_t *__restrict__ tokens, const float *state_in,
                                                        float *state_out, float *__restrict__ logits,
                                                        int32_t *__restrict__ experts, int *__restrict__ bad,
                                                        unsigned *__restrict__ stats) {
    constexpr int NT = N * TPR, NW = NT / 32;
    static_assert(TPR == 1 || TPR == 4, "the parts of a coordinate's sums are added as four");
    __shared__ float hp[TPR == 1 ? N : 1], below[N], vv[N], vpart[NT], emb[N], red[NW * 32], sums[32], bsh[2][16];
    __shared__ float zs[kMaxLayers][32];
    __shared__ int nodesh;
    __shared__ float rmsq;   // small batches: sum of h^2 of the layer
    __shared__ float hs[TPR > 1 ? kMaxLayers * N : 1];   // small batches: the stream's state of every layer, read at once
    __shared__ float es[TPR > 1 ? kMaxLayers * 32 : 1];  // and the token's router embedding of every layer (F <= 32)
    extern __shared__ __align__(16) float vts[];          // V' of the next routed layer, when staged (vsm)
    __shared__ __align__(8) uint64_t vbar;                 // its copy's mbarrier
    // thread t: coordinate row, part sub of its sums; with TPR > 1 the parts are quarters of the block (a warp holds 32
    // consecutive coordinates of one part, so that its loads of an expert row are one line), added in shared memory
    const int t = threadIdx.x, row = TPR > 1 ? t % N : t, sub = TPR > 1 ? t / N : 0;
    __shared__ float xq[TPR > 1 ? TPR * N : 1];   // the TPR parts of a sum per coordinate
    const int L = m.L, V = m.V, C = m.C, R = m.R, R2 = m.R2, F = m.F, FIN = m.FIN, bsz = m.b;
    const int SW = N / 16 + 1 + R;
    if constexpr (TPR > 1) {   // a batch of a few streams, each step a chain of dependent loads: the arrays every
        // stream reads (the routed layers' router rows, V' and Q) are prefetched into L2 at once, so that the router
        // rounds and the layer inputs hit L2 rather than wait on DRAM. The pieces are shared out over the helper
        // blocks past the streams' (an SM's bulk copies run one after another, and a stream's own loads would queue
        // behind them), or over the whole grid when there are none.
        const int H = gridDim.x > B ? gridDim.x - B : 0;
        if (H == 0 || blockIdx.x >= B) {
            const unsigned g = (H > 0 ? blockIdx.x - B : blockIdx.x) * NT + t, G = (H > 0 ? H : gridDim.x) * NT;
            for (int l = 1; l < L; l++) {
                const FLayer &y = m.layer[l];
                size_t wbn = 0;   // the round-blocked router rows, which the small-batch router reads
                for (int d0 = 0; d0 < m.D; d0 += kLook) wbn += ((size_t)FIN << d0) << min(kLook, m.D - d0);
                prefetch_spread(y.wb, wbn, g, G);
                if (y.vt != nullptr) prefetch_spread(y.vt, (size_t)N * R2, g, G);
            }
            for (int l = 0; l < L; l++) prefetch_spread(m.layer[l].qt, (size_t)R * C, g, G);
        }
    }
    // a batch of a few streams: V' of each routed layer is copied into shared memory (the launch gives the dynamic
    // shared memory) while the layer below finishes, by one bulk copy that thread 0 issues; every thread waits for its
    // phase, with a limit after which the launch reports YGG_E_TIMEOUT and the block reads V' from global memory
    bool vsm = TPR > 1 && R2 > 0 && N * R2 <= kVtSmem;
    unsigned vphase = 0;
    if (vsm) {
        if (t == 0) {
            asm volatile("mbarrier.init.shared.b64 [%0], 1;" ::"r"((unsigned)__cvta_generic_to_shared(&vbar)));
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
    }
    auto stage_vt = [&](const float *vt) {
        if (t == 0) bulk_to_shared(vts, vt, (uint32_t)(N * R2 * sizeof(float)), &vbar);
    };
    for (int s = blockIdx.x; s < B; s += gridDim.x) {
        const int x = tokens[s];
        if (x < 0 || x >= V) {   // the whole stream is skipped: NaN logits, state unchanged
            if (t == 0) atomicOr(bad, 1);
            for (int c = t; c < C; c += NT) logits[(size_t)s * C + c] = __int_as_float(0x7fc00000);
            for (int i = t; i < L * N; i += NT) state_out[(size_t)s * L * N + i] = state_in[(size_t)s * L * N + i];
            if (experts != nullptr && t < L) experts[(size_t)s * L + t] = -1;
            continue;
        }
        // with TPR > 1 and at most n classes, the head is added layer by layer at the readout (thread (row, sub) holding
        // class row's sum over the rows k = sub mod TPR); otherwise it follows the last layer
        const bool head_in_layers = TPR > 1 && C <= N;
        float lgp = 0.0f;
        if constexpr (TPR > 1) {   // the stream's state in, every layer's at once (published by layer 0's barrier)
            for (int i = t; i < L * N; i += NT) hs[i] = state_in[(size_t)s * L * N + i];
            if (F <= 32)
                for (int i = t; i < (L - 1) * 32; i += NT)
                    if (i % 32 < F) es[i] = __ldg(m.layer[1 + i / 32].embed + (size_t)x * F + i % 32);
        }
        for (int l = 0; l < L; l++) {
            const FLayer &y = m.layer[l];
            if constexpr (TPR == 1) hp[row] = state_in[((size_t)s * L + l) * N + row];
            const float *hpl = TPR > 1 ? hs + l * N : hp;   // h of this layer before the step
            int r = x;
            if (l > 0) {
                if (t < F) emb[t] = TPR > 1 && F <= 32 ? es[(l - 1) * 32 + t] : __ldg(y.embed + (size_t)x * F + t);
                // layer input v = V' rms(h_below): the n inputs split into NP parts, thread (part, k) sums its part of
                // row k, then thread k adds the parts. With TPR > 1 and V' in shared memory, the threads past the
                // routing warps' do it while those route and add the parts among themselves (vsplit); otherwise every
                // thread does, before the router, reading V' from global memory.
                if constexpr (TPR > 1) {
                    if (vsm) {
                        if (!wait_phase(&vbar, vphase)) {   // V' did not land: report, and read it from global memory
                            atomicOr(bad, 2);
                            vsm = false;
                        }
                        vphase ^= 1;
                    }
                }
                const int RWT = TPR > 1 ? (FIN + 31) / 32 * 32 : 0;   // the routing threads
                int NP = R2 > 0 ? max(1, NT / R2) : 1, span = (N + NP - 1) / NP;   // the unsplit parts
                // hs, emb, V'; below was written before the last barrier of the layer below. The vote makes the
                // outcome of the V' wait the block's, so that the split and its barrier below are uniform.
                if constexpr (TPR > 1) vsm = __syncthreads_and(vsm);
                else __syncthreads();
                const bool vsplit = vsm && R2 <= NT - RWT;
                const int vb = vsplit ? RWT : 0, vi = t - vb;
                if (vsplit) { NP = max(1, (NT - vb) / R2); span = (N + NP - 1) / NP; }
                const bool vpart_on = y.vt != nullptr && vi >= 0 && vi < NP * R2;
                const int k = R2 > 0 && vi >= 0 ? vi % R2 : 0, i0 = (vi >= 0 ? vi / max(R2, 1) : 0) * span,
                          i1 = min(N, i0 + span);
                auto layer_input_part = [&]() {
                    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                    if (vsm) {
                        int i = i0;
#pragma unroll 4
                        for (; i + 3 < i1; i += 4) {
                            a0 = fmaf(vts[i * R2 + k], below[i], a0);
                            a1 = fmaf(vts[(i + 1) * R2 + k], below[i + 1], a1);
                            a2 = fmaf(vts[(i + 2) * R2 + k], below[i + 2], a2);
                            a3 = fmaf(vts[(i + 3) * R2 + k], below[i + 3], a3);
                        }
                        for (; i < i1; i++) a0 = fmaf(vts[i * R2 + k], below[i], a0);
                    } else {
                        int i = i0;
#pragma unroll(TPR > 1 ? 4 : 1)
                        for (; i + 3 < i1; i += 4) {
                            a0 = fmaf(__ldg(y.vt + (size_t)i * R2 + k), below[i], a0);
                            a1 = fmaf(__ldg(y.vt + (size_t)(i + 1) * R2 + k), below[i + 1], a1);
                            a2 = fmaf(__ldg(y.vt + (size_t)(i + 2) * R2 + k), below[i + 2], a2);
                            a3 = fmaf(__ldg(y.vt + (size_t)(i + 3) * R2 + k), below[i + 3], a3);
                        }
                        for (; i < i1; i++) a0 = fmaf(__ldg(y.vt + (size_t)i * R2 + k), below[i], a0);
                    }
                    vpart[vi] = (a0 + a1) + (a2 + a3);
                };
                if (vpart_on && !vsplit) layer_input_part();
                // router: rounds of kLook levels, node j (0-based heap) right iff f . W_j + b_j > 0; thread t takes the
                // features t, t + NT, ... of f = [router_embed(x); rms(h_below)]
                float f0 = 0.0f, f1 = 0.0f;
                if (t < FIN) f0 = t < F ? emb[t] : below[t - F];
                if (t + NT < FIN) f1 = t + NT < F ? emb[t + NT] : below[t + NT - F];
                int node = 0;
                if constexpr (TPR > 1) {
                    // a batch of a few streams: only the RW warps that hold a feature route (thread t < F + n, one
                    // feature each), so that a round costs them their loads and one short barrier rather than the
                    // block's 32 warps' issue. Thread t reads its feature's weights of the round's rows from the
                    // round-blocked copy (16-byte loads that coalesce over the warp), each warp reduce-scatters its 15
                    // partial sums into red, and after a named barrier every routing warp adds the warps' sums and
                    // walks the round itself (same order, same node). red and the biases alternate by round parity,
                    // so the next round's writes never meet this round's reads. The other warps meanwhile sum the
                    // layer input (vsplit), then wait for the node.
                    const int RW = (FIN + 31) / 32, lane = t & 31;
                    if (t < RW * 32) {
                        size_t woff = 0;   // the round's first block in wb
                        for (int d0 = 0; d0 < m.D; d0 += kLook) {
                            const int lv = min(kLook, m.D - d0), P = 1 << lv;
                            const int nrows = P - 1, par = (d0 / kLook) & 1;
                            if (t < nrows) bsh[par][t] = __ldg(y.bias + node * (1 << (31 - __clz(t + 1))) + t);
                            const float *blk = y.wb + woff + (size_t)(node - ((1 << d0) - 1)) * FIN * P;
                            float wv[16];
#pragma unroll
                            for (int q = 0; q < 4; q++) {
                                float4 v4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                                if (t < FIN && 4 * q < P) {
                                    if (P >= 4) v4 = __ldg(reinterpret_cast<const float4 *>(blk) + (size_t)q * FIN + t);
                                    else v4.x = __ldg(blk + 2 * t);   // P = 2: the round's one row
                                }
                                wv[4 * q] = v4.x; wv[4 * q + 1] = v4.y; wv[4 * q + 2] = v4.z; wv[4 * q + 3] = v4.w;
                            }
                            float part[16];
#pragma unroll
                            for (int k = 0; k < 16; k++) part[k] = k < nrows ? wv[k] * f0 : 0.0f;
                            const float rs = reduce_scatter<16>(part, lane);   // lanes 2k, 2k + 1: this warp's row k
                            float *rd = red + par * (NW * 16);
                            if ((lane & 1) == 0) rd[(t >> 5) * 16 + (lane >> 1)] = rs;
                            named_sync(1, RW * 32);
                            float a = 0.0f;   // lane k < nrows: row k over the warps, and its bias
                            if (lane < nrows) {
#pragma unroll
                                for (int w = 0; w < 16; w++)   // RW <= 16 (F + n <= 2 n <= 512)
                                    if (w < RW) a += rd[w * 16 + lane];
                                a += bsh[par][lane];
                            }
                            const unsigned dec = __ballot_sync(kFull, lane < nrows && a > 0.0f);   // bit k: row k right
                            int rr = 0;
                            for (int j = 0; j < lv; j++) rr = 2 * rr + 1 + (int)((dec >> rr) & 1u);
                            node = node * (1 << lv) + rr;
                            woff += ((size_t)FIN << d0) * P;
                        }
                        if (t == 0) nodesh = node;
                    } else if (vsplit) {   // the other warps: the layer input's parts, then their sum
                        if (vpart_on) layer_input_part();
                        named_sync(2, NT - RWT);
                        if (vi < R2) {
                            float a = 0.0f;
                            for (int q = 0; q < NP; q++) a += vpart[q * R2 + vi];
                            vv[vi] = a;
                        }
                    }
                    __syncthreads();   // the node; v (V' in shared memory is read no more in this layer)
                    node = nodesh;
                } else {
                for (int d0 = 0; d0 < m.D; d0 += kLook) {
                    const int lv = min(kLook, m.D - d0);
                    const int nrows = (1 << lv) - 1;
                    // the rows' loads first (rows past the round's levels read the current node's row, unused), then
                    // the products: a load used inside its own branch would stall the warp once per row. Thread k < 15
                    // loads row k's bias into shared memory meanwhile.
                    float *bs = bsh[(d0 / kLook) & 1];   // by round parity: the last round's walk may still read the other
                    if (t < nrows) bs[t] = __ldg(y.bias + node * (1 << (31 - __clz(t + 1))) + t);
                    float wv[16];
#pragma unroll
                    for (int k = 0; k < 16; k++) {
                        const int lvl = k == 0 ? 0 : k < 3 ? 1 : k < 7 ? 2 : 3;
                        const int nd = k < nrows ? node * (1 << lvl) + k : node;
                        wv[k] = t < FIN ? __ldg(y.w + (size_t)nd * FIN + t) : 0.0f;
                    }
                    float part[16];
#pragma unroll
                    for (int k = 0; k < 16; k++) part[k] = k < nrows ? wv[k] * f0 : 0.0f;
                    if constexpr (TPR == 1) {   // n threads, F + n features: the last F features a second time
                        if (t + NT < FIN) {
#pragma unroll
                            for (int k = 0; k < 16; k++) {
                                const int lvl = k == 0 ? 0 : k < 3 ? 1 : k < 7 ? 2 : 3;
                                const int nd = k < nrows ? node * (1 << lvl) + k : node;
                                wv[k] = __ldg(y.w + (size_t)nd * FIN + t + NT);
                            }
#pragma unroll
                            for (int k = 0; k < 16; k++)
                                if (k < nrows) part[k] = fmaf(wv[k], f1, part[k]);
                        }
                    }
                    block_sum<16, NW>(part, red, sums, t);
                    int rr = 0;
                    for (int j = 0; j < lv; j++) rr = 2 * rr + 1 + (sums[rr] + bs[rr] > 0.0f ? 1 : 0);
                    node = node * (1 << lv) + rr;
                }
                }
                r = node - ((1 << m.D) - 1);
                // the chosen expert's arrays towards L2 (without the split, while the layer input's parts are added):
                // at small batches one 128-byte line per thread (the requests leave at once, over the whole block),
                // else one bulk prefetch per array
                if constexpr (TPR > 1) {
                    const int lt = N / 32, lu = y.ut != nullptr ? R2 * N / 32 : 0, la = y.at != nullptr ? bsz * N / 32 : 0;
                    for (int i = t; i < lt + lu + la + R * N / 32; i += NT) {
                        const float *a = i < lt ? y.table + ((size_t)r * V + x) * N + 32 * i
                                       : i < lt + lu ? y.ut + (size_t)r * R2 * N + 32 * (i - lt)
                                       : i < lt + lu + la ? y.at + (size_t)r * bsz * N + 32 * (i - lt - lu)
                                       : y.pt + (size_t)r * R * N + 32 * (i - lt - lu - la);
                        asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
                    }
                } else {
                    if (t == 0) prefetch_l2(y.table + ((size_t)r * V + x) * N, N * 4u);
                    if (t == 32 && y.ut != nullptr) prefetch_l2(y.ut + (size_t)r * R2 * N, (uint32_t)R2 * N * 4u);
                    if (t == 64 % NT && y.at != nullptr) prefetch_l2(y.at + (size_t)r * bsz * N, (uint32_t)bsz * N * 4u);
                    if (t == 96 % NT) prefetch_l2(y.pt + (size_t)r * R * N, (uint32_t)R * N * 4u);
                }
                if (!vsplit) {
                    if (y.vt != nullptr && t < R2) {
                        float a = 0.0f;
                        for (int q = 0; q < NP; q++) a += vpart[q * R2 + t];
                        vv[t] = a;
                    }
                    __syncthreads();   // vv
                }
                if (stats != nullptr && y.vt != nullptr) {
                    float a = t < R2 ? fabsf(vv[t]) : 0.0f;
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(kFull, a, off));
                    if ((t & 31) == 0 && t < R2) max_into(stats + (size_t)l * SW + N / 16, a);
                }
            } else {
                __syncthreads();   // hp
            }
            // this thread's readout rows of P_r (k = sub mod TPR), loaded with the expert's other arrays when a
            // thread holds few of them (TPR > 1); with one thread per coordinate they are loaded at the readout, as
            // 32 more live registers would cost the large batches their occupancy
            constexpr int kPV = TPR > 1 ? RP / TPR : 1;
            float pv[kPV > 0 ? kPV : 1];
            const float *p = y.pt + (size_t)r * R * N + row;
            float qv[kPV > 0 ? kPV : 1];   // Q_l[k][class row], k = sub mod TPR, when the head is added here
            if constexpr (TPR > 1) {
#pragma unroll
                for (int j = 0; j < RP / TPR; j++) {
                    const int k = j * TPR + sub;
                    pv[j] = k < R ? __ldg(p + (size_t)k * N) : 0.0f;
                    qv[j] = head_in_layers && k < R && row < C ? __ldg(y.qt + (size_t)k * C + row) : 0.0f;
                }
            }
            // h = T_r[x] + U'_r v + A_r h_prev: each of the TPR threads of a coordinate sums every TPR-th term
            float h = sub == 0 ? __ldg(y.table + (l == 0 ? (size_t)x * N : ((size_t)r * V + x) * N) + row) : 0.0f;
            if (l > 0 && y.ut != nullptr) {
                const float *u = y.ut + (size_t)r * R2 * N + row;
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                int k = sub;
#pragma unroll(TPR > 1 ? 4 : 2)
                for (; k + 3 * TPR < R2; k += 4 * TPR) {
                    a0 = fmaf(__ldg(u + (size_t)k * N), vv[k], a0);
                    a1 = fmaf(__ldg(u + (size_t)(k + TPR) * N), vv[k + TPR], a1);
                    a2 = fmaf(__ldg(u + (size_t)(k + 2 * TPR) * N), vv[k + 2 * TPR], a2);
                    a3 = fmaf(__ldg(u + (size_t)(k + 3 * TPR) * N), vv[k + 3 * TPR], a3);
                }
                for (; k < R2; k += TPR) a0 = fmaf(__ldg(u + (size_t)k * N), vv[k], a0);
                h += (a0 + a1) + (a2 + a3);
            }
            if (y.at != nullptr) {
                const float *a = y.at + (size_t)r * bsz * N + row;
                const int blk0 = (row / bsz) * bsz;
                float a0 = 0.0f, a1 = 0.0f;
                if constexpr (TPR > 1) {
                    constexpr int kA = 32 / TPR;   // block size <= 32: this thread's columns j = sub mod TPR, loaded first
                    float av[kA];
#pragma unroll
                    for (int jj = 0; jj < kA; jj++) {
                        const int j = jj * TPR + sub;
                        av[jj] = j < bsz ? __ldg(a + (size_t)j * N) : 0.0f;
                    }
#pragma unroll
                    for (int jj = 0; jj < kA; jj += 2) {
                        const int j = jj * TPR + sub;
                        if (j < bsz) a0 = fmaf(av[jj], hpl[blk0 + j], a0);
                        if (jj + 1 < kA && j + TPR < bsz) a1 = fmaf(av[jj + 1], hpl[blk0 + j + TPR], a1);
                    }
                } else {
#pragma unroll 4
                    for (int j = 0; j < bsz; j += 2) {
                        a0 = fmaf(__ldg(a + (size_t)j * N), hpl[blk0 + j], a0);
                        if (j + 1 < bsz) a1 = fmaf(__ldg(a + (size_t)(j + 1) * N), hpl[blk0 + j + 1], a1);
                    }
                }
                h += a0 + a1;
            }
            if constexpr (TPR > 1) {   // the parts of h, in a fixed order (every part's thread gets the same h)
                xq[sub * N + row] = h;
                __syncthreads();
                h = (xq[row] + xq[N + row]) + (xq[2 * N + row] + xq[3 * N + row]);
            }
            if (sub == 0) state_out[((size_t)s * L + l) * N + row] = h;
            if (vsm && l + 1 < L) stage_vt(m.layer[l + 1].vt);   // the next layer's V', while this one finishes
            if (experts != nullptr && t == 0) experts[(size_t)s * L + l] = r;
            if (stats != nullptr) {   // group maxima of |h|, a warp's share of each group of 16 coordinates at a time
                float a = fabsf(h);
#pragma unroll
                for (int off = 1; off < 16; off <<= 1) a = fmaxf(a, __shfl_xor_sync(kFull, a, off));
                if (sub == 0 && (t & 15) == 0) max_into(stats + (size_t)l * SW + row / 16, a);
            }
            // readout z = P_r h (thread sub takes the rows k = sub mod TPR), and sum h^2 for rms(h)
            if constexpr (TPR > 1) {
                // a warp holds one part sub (rows k = 4 j + sub): it reduce-scatters its KQ sums into red, its h^2 too
                // when sub = 0; after one barrier warp 0 adds the NWS warps of each part and the h^2 sums (fixed
                // orders), and after a second every thread has z and rms(h)
                constexpr int KQ = RP / TPR > 1 ? RP / TPR : 2, NWS = N / 32, LKQ = Log2<KQ>::value;
                const int lane = t & 31, warp = t >> 5;
                float pq[KQ];
#pragma unroll
                for (int j = 0; j < KQ; j++) pq[j] = j < RP / TPR ? pv[j] * h : 0.0f;
                const float rsum = reduce_scatter<KQ>(pq, lane);   // lane l: this warp's sum of pq[l >> (5 - LKQ)]
                if ((lane & ((32 >> LKQ) - 1)) == 0) red[warp * KQ + (lane >> (5 - LKQ))] = rsum;
                if (sub == 0) {
                    float q = h * h;
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(kFull, q, off);
                    if (lane == 0) red[NW * KQ + warp] = q;
                }
                __syncthreads();
                if (t < 32) {
                    float z = 0.0f;
                    if (lane < R) {
                        const int ks = lane % TPR, kj = lane / TPR;
#pragma unroll
                        for (int w = 0; w < NWS; w++) z += red[(ks * NWS + w) * KQ + kj];
                        sums[lane] = z;
                        zs[l][lane] = z;
                        if (stats != nullptr) max_into(stats + (size_t)l * SW + N / 16 + 1 + lane, z);
                    }
                    if (lane == 0) {
                        float q = 0.0f;
#pragma unroll
                        for (int w = 0; w < NWS; w++) q += red[NW * KQ + w];
                        rmsq = q;
                    }
                }
                __syncthreads();
                if (head_in_layers) {
#pragma unroll
                    for (int j = 0; j < RP / TPR; j++)
                        if (j * TPR + sub < R) lgp = fmaf(sums[j * TPR + sub], qv[j], lgp);
                }
                if (sub == 0) below[row] = h * rsqrtf(rmsq / (float)N + kRmsEps);
            } else {
                float part[RP];
#pragma unroll
                for (int k = 0; k < RP; k++) {
                    if constexpr (TPR > 1) part[k] = (k % TPR == sub) ? pv[k / TPR] * h : 0.0f;
                    else part[k] = k < R ? __ldg(p + (size_t)k * N) * h : 0.0f;
                }
                block_sum<RP, NW>(part, red, sums, t);
                if (t < R) {
                    zs[l][t] = sums[t];
                    if (stats != nullptr) max_into(stats + (size_t)l * SW + N / 16 + 1 + t, sums[t]);
                }
                float sq[1] = {sub == 0 ? h * h : 0.0f};
                block_sum<1, NW>(sq, red, sums, t);
                if (sub == 0) below[row] = h * rsqrtf(sums[0] / (float)N + kRmsEps);
            }
            __syncthreads();   // below, zs
        }
        if (head_in_layers) {   // logits = output_bias + the TPR threads' sums of class row
            xq[sub * N + row] = lgp;   // (the last use of xq, h's parts, was before the readout's barriers)
            __syncthreads();
            if (row < C && sub == 0)
                logits[(size_t)s * C + row] =
                    __ldg(m.out_bias + row) + ((xq[row] + xq[N + row]) + (xq[2 * N + row] + xq[3 * N + row]));
        }
        // logits = output_bias + sum_l z_l Q_l^T: TPR threads per class, thread sub taking the layers l = sub mod TPR
        // (a layer's R unembedding loads issued together), then added over the TPR threads
        for (int c0 = 0; c0 < (head_in_layers ? 0 : C); c0 += N) {
            const int c = c0 + row;
            float lg = 0.0f;
            if (c < C) {
                for (int l = sub; l < L; l += TPR) {
                    const float *q = m.layer[l].qt + c;
                    float qv[RP];
#pragma unroll
                    for (int k = 0; k < RP; k++) qv[k] = k < R ? __ldg(q + (size_t)k * C) : 0.0f;
#pragma unroll
                    for (int k = 0; k < RP; k++)
                        if (k < R) lg = fmaf(zs[l][k], qv[k], lg);
                }
            }
            if constexpr (TPR > 1) {
                xq[sub * N + row] = lg;
                __syncthreads();
                if (c < C && sub == 0)
                    logits[(size_t)s * C + c] =
                        __ldg(m.out_bias + c) + ((xq[row] + xq[N + row]) + (xq[2 * N + row] + xq[3 * N + row]));
                __syncthreads();   // xq before the next classes
            } else {
                if (c < C) logits[(size_t)s * C + c] = __ldg(m.out_bias + c) + lg;
            }
        }
        __syncthreads();   // zs, hp before the next stream
    }
}

}  // namespace fstep
}  // namespace ygg

using namespace ygg::fstep;

struct ygg_fmodel {
    int device;
    FModel dm;
    ygg_fshape_t shape;
    float *d_blob;
    int *d_bad;
    int sm_count;
};

namespace {

size_t align_floats(size_t x) { return (x + 63) / 64 * 64; }   // 256-byte aligned sub-arrays

template <int N, int RP, int TPR>
cudaError_t launch_t(const FModel &dm, int B, const int32_t *tok, const float *sin, float *sout, float *lg, int32_t *ex,
                     int *bad, unsigned *stats, int grid, cudaStream_t st) {
    // the small-batch instances stage V' in dynamic shared memory (the kernel's vsm)
    const size_t dyn = TPR > 1 && dm.R2 > 0 && N * dm.R2 <= kVtSmem ? (size_t)N * dm.R2 * sizeof(float) : 0;
    if (dyn > 0) {
        static bool opted[64] = {};   // per device: the opt-in above the default 48 KB
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64 || !opted[dev]) {
            const cudaError_t e = cudaFuncSetAttribute(fstep_kernel<N, RP, TPR>,
                                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kVtSmem * 4);
            if (e != cudaSuccess) return e;
            if (dev >= 0 && dev < 64) opted[dev] = true;
        }
    }
    fstep_kernel<N, RP, TPR><<<grid, N * TPR, dyn, st>>>(dm, B, tok, sin, sout, lg, ex, bad, stats);
    return cudaGetLastError();
}

template <int N, int TPR>
cudaError_t launch_n(const FModel &dm, int B, const int32_t *tok, const float *sin, float *sout, float *lg, int32_t *ex,
                     int *bad, unsigned *stats, int grid, cudaStream_t st) {
    if (dm.R <= 8) return launch_t<N, 8, TPR>(dm, B, tok, sin, sout, lg, ex, bad, stats, grid, st);
    if (dm.R <= 16) return launch_t<N, 16, TPR>(dm, B, tok, sin, sout, lg, ex, bad, stats, grid, st);
    return launch_t<N, 32, TPR>(dm, B, tok, sin, sout, lg, ex, bad, stats, grid, st);
}

// TPR = 4 threads per coordinate for a batch of at most two streams per SM (each stream's loads spread over 4x the
// threads: its step is a chain of dependent loads), 1 above (more streams per SM, fewer reductions)
template <int N>
cudaError_t launch_tpr(const FModel &dm, int B, const int32_t *tok, const float *sin, float *sout, float *lg,
                       int32_t *ex, int *bad, unsigned *stats, int sm_count, cudaStream_t st) {
    // up to 32 helper blocks that only prefetch, while SMs are left over
    if (B <= 2 * sm_count)
        return launch_n<N, 4>(dm, B, tok, sin, sout, lg, ex, bad, stats, B + std::max(0, std::min(32, sm_count - B)), st);
    const int grid = B < 32 * sm_count ? B : 32 * sm_count;
    return launch_n<N, 1>(dm, B, tok, sin, sout, lg, ex, bad, stats, grid, st);
}

}  // namespace

extern "C" {

int ygg_fload(const ygg_fshape_t *sh, const float *const *arrays, int device, ygg_fmodel **out) {
    if (!sh || !arrays || !out) return YGG_E_ARG;
    *out = nullptr;
    const int L = sh->n_layers, n = sh->d_state, b = sh->block_size, V = sh->vocab, C = sh->classes;
    const int D = sh->router_depth, F = sh->router_token_dim, R = sh->readout_rank, R2 = sh->layer_input_rank;
    if (L < 2 || L > kMaxLayers || (n != 64 && n != 128 && n != 256) || b < 2 || b > 32 || (b & 1) || n % b ||
        V < 1 || C < 1 || D < 1 || D > 20 || F < 1 || F > n || R < 1 || R > 32 || R2 < 0 || R2 > n)
        return YGG_E_UNSUPPORTED;
    const int E = 1 << D, FIN = F + (sh->route_on_state ? n : 0);
    for (int l = 0; l < L; l++) {
        const float *const *a = arrays + (size_t)l * YGG_F_ARRAYS_PER_LAYER;
        if (!a[0] || !a[2] || !a[3]) return YGG_E_MISSING;
        if ((l == 0 ? sh->token_transition : sh->routed_transition) && !a[1]) return YGG_E_MISSING;
        if (l > 0 && (!a[4] || !a[5] || !a[6] || (R2 > 0 && (!a[7] || !a[8])))) return YGG_E_MISSING;
    }
    if (!arrays[(size_t)L * YGG_F_ARRAYS_PER_LAYER]) return YGG_E_MISSING;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return YGG_E_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) return YGG_E_DEVICE;
    // host staging of the device layout: one blob, every sub-array 256-byte aligned
    std::vector<float> blob;
    auto take = [&](size_t count) {
        const size_t off = blob.size();
        blob.resize(off + align_floats(count), 0.0f);
        return off;
    };
    struct Off { size_t table, at, pt, qt, embed, w, bias, wb, vt, ut; bool has_at, has_v; };
    std::vector<Off> offs(L);
    for (int l = 0; l < L; l++) {
        const float *const *a = arrays + (size_t)l * YGG_F_ARRAYS_PER_LAYER;
        const bool tok = l == 0;
        const size_t Ex = tok ? (size_t)V : (size_t)E;
        Off &o = offs[l];
        // table: token layer its own rows T_x[x] (V, n); routed (E, V, n)
        const size_t tcount = tok ? (size_t)V * n : (size_t)E * V * n;
        o.table = take(tcount);
        memcpy(blob.data() + o.table, a[0], tcount * sizeof(float));
        o.has_at = (tok ? sh->token_transition : sh->routed_transition) != 0;
        if (o.has_at) {   // (E, n/b, b, b) -> (E, b, n)
            o.at = take(Ex * b * n);
            for (size_t e = 0; e < Ex; e++)
                for (int i = 0; i < n; i++)
                    for (int j = 0; j < b; j++)
                        blob[o.at + (e * b + j) * n + i] = a[1][((e * (n / b) + i / b) * b + i % b) * b + j];
        }
        o.pt = take(Ex * R * n);
        memcpy(blob.data() + o.pt, a[2], Ex * R * n * sizeof(float));
        o.qt = take((size_t)R * C);   // (C, R) -> (R, C)
        for (int c = 0; c < C; c++)
            for (int k = 0; k < R; k++) blob[o.qt + (size_t)k * C + c] = a[3][(size_t)c * R + k];
        o.has_v = false;
        if (!tok) {
            o.embed = take((size_t)V * F);
            memcpy(blob.data() + o.embed, a[4], (size_t)V * F * sizeof(float));
            o.w = take((size_t)(E - 1) * FIN);
            memcpy(blob.data() + o.w, a[5], (size_t)(E - 1) * FIN * sizeof(float));
            o.bias = take(E - 1);
            memcpy(blob.data() + o.bias, a[6], (size_t)(E - 1) * sizeof(float));
            size_t wbn = 0;   // the round-blocked copy of the rows (FLayer::wb)
            for (int d0 = 0; d0 < D; d0 += kLook) wbn += ((size_t)FIN << d0) << std::min(kLook, D - d0);
            o.wb = take(wbn);
            size_t woff = o.wb;
            for (int d0 = 0; d0 < D; d0 += kLook) {
                const int lv = std::min(kLook, D - d0), P = 1 << lv;
                for (size_t mi = 0; mi < ((size_t)1 << d0); mi++) {
                    const size_t root = ((size_t)1 << d0) - 1 + mi;
                    for (int k = 0; k < P - 1; k++) {
                        int lvl = 0;
                        while ((2 << lvl) - 1 <= k) lvl++;   // the level of local row k: 2^lvl - 1 <= k < 2^(lvl+1) - 1
                        const size_t nd = (root << lvl) + k;
                        const size_t blk = woff + (size_t)mi * FIN * P;
                        for (int f = 0; f < FIN; f++)
                            blob[P >= 4 ? blk + ((size_t)(k / 4) * FIN + f) * 4 + k % 4 : blk + (size_t)f * 2 + k] =
                                a[5][nd * FIN + f];
                    }
                }
                woff += ((size_t)FIN << d0) * P;
            }
            o.has_v = R2 > 0;
            if (o.has_v) {
                o.vt = take((size_t)n * R2);   // (R2, n) -> (n, R2)
                for (int k = 0; k < R2; k++)
                    for (int i = 0; i < n; i++) blob[o.vt + (size_t)i * R2 + k] = a[7][(size_t)k * n + i];
                o.ut = take((size_t)E * R2 * n);   // (E, n, R2) -> (E, R2, n)
                for (size_t e = 0; e < (size_t)E; e++)
                    for (int i = 0; i < n; i++)
                        for (int k = 0; k < R2; k++)
                            blob[o.ut + (e * R2 + k) * n + i] = a[8][(e * n + i) * R2 + k];
            }
        }
    }
    const size_t ob = take(C);
    memcpy(blob.data() + ob, arrays[(size_t)L * YGG_F_ARRAYS_PER_LAYER], (size_t)C * sizeof(float));

    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return YGG_E_DEVICE;
    ygg_fmodel *m = new ygg_fmodel();
    m->device = device;
    m->shape = *sh;
    m->sm_count = prop.multiProcessorCount;
    int rc = YGG_OK;
    if (cudaMalloc((void **)&m->d_blob, blob.size() * sizeof(float)) != cudaSuccess ||
        cudaMalloc((void **)&m->d_bad, sizeof(int)) != cudaSuccess) {
        rc = YGG_E_OOM;
    } else if (cudaMemcpy(m->d_blob, blob.data(), blob.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
               cudaMemset(m->d_bad, 0, sizeof(int)) != cudaSuccess) {
        rc = YGG_E_CUDA;
    }
    if (rc != YGG_OK) {
        cudaFree(m->d_blob);
        cudaFree(m->d_bad);
        delete m;
        if (prev >= 0) cudaSetDevice(prev);
        return rc;
    }
    FModel &dm = m->dm;
    memset(&dm, 0, sizeof dm);
    dm.L = L; dm.n = n; dm.b = b; dm.V = V; dm.C = C; dm.D = D; dm.F = F; dm.FIN = FIN; dm.R = R; dm.R2 = R2;
    dm.route_on_state = sh->route_on_state != 0;
    const float *d = m->d_blob;
    dm.out_bias = d + ob;
    for (int l = 0; l < L; l++) {
        const Off &o = offs[l];
        FLayer &y = dm.layer[l];
        y.table = d + o.table;
        y.at = o.has_at ? d + o.at : nullptr;
        y.pt = d + o.pt;
        y.qt = d + o.qt;
        if (l > 0) {
            y.embed = d + o.embed;
            y.w = d + o.w;
            y.bias = d + o.bias;
            y.wb = d + o.wb;
            y.vt = o.has_v ? d + o.vt : nullptr;
            y.ut = o.has_v ? d + o.ut : nullptr;
        }
    }
    if (prev >= 0) cudaSetDevice(prev);
    *out = m;
    return YGG_OK;
}

int ygg_fstep_stats(const ygg_fmodel *m, int batch, const int32_t *d_tokens, const float *d_state_in,
                    float *d_state_out, float *d_logits, int32_t *d_experts, float *d_stats, void *stream) {
    if (!m || batch < 0) return YGG_E_ARG;
    if (batch == 0) return YGG_OK;
    if (!d_tokens || !d_state_in || !d_state_out || !d_logits) return YGG_E_ARG;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != m->device && cudaSetDevice(m->device) != cudaSuccess) return YGG_E_CUDA;
    const FModel &dm = m->dm;
    // a block per stream, streams beyond the grid in a grid-stride loop (launch_tpr picks the block shape)
    const cudaStream_t st = (cudaStream_t)stream;
    unsigned *stats = (unsigned *)d_stats;
    const int sm = m->sm_count;
    cudaError_t e;
    switch (dm.n) {
        case 64: e = launch_tpr<64>(dm, batch, d_tokens, d_state_in, d_state_out, d_logits, d_experts, m->d_bad, stats, sm, st); break;
        case 128: e = launch_tpr<128>(dm, batch, d_tokens, d_state_in, d_state_out, d_logits, d_experts, m->d_bad, stats, sm, st); break;
        default: e = launch_tpr<256>(dm, batch, d_tokens, d_state_in, d_state_out, d_logits, d_experts, m->d_bad, stats, sm, st); break;
    }
    if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
    return e == cudaSuccess ? YGG_OK : YGG_E_CUDA;
}

int ygg_fstep(const ygg_fmodel *m, int batch, const int32_t *d_tokens, const float *d_state_in, float *d_state_out,
              float *d_logits, int32_t *d_experts, void *stream) {
    return ygg_fstep_stats(m, batch, d_tokens, d_state_in, d_state_out, d_logits, d_experts, nullptr, stream);
}

int ygg_fstatus(const ygg_fmodel *m, void *stream, int *status_out) {
    if (!m || !status_out) return YGG_E_ARG;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != m->device && cudaSetDevice(m->device) != cudaSuccess) return YGG_E_CUDA;
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, m->d_bad, sizeof v, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e == cudaSuccess && v) e = cudaMemsetAsync(m->d_bad, 0, sizeof(int), (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
    if (e != cudaSuccess) return YGG_E_CUDA;
    *status_out = (v & 2) ? YGG_E_TIMEOUT : v ? YGG_E_TOKEN : YGG_OK;
    return YGG_OK;
}

void ygg_ffree(ygg_fmodel *m) {
    if (!m) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    cudaFree(m->d_blob);
    cudaFree(m->d_bad);
    if (prev >= 0) cudaSetDevice(prev);
    delete m;
}

}  // extern "C"
