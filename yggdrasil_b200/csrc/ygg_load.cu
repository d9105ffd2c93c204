// The C-ABI of libygg_b200: YGG1 parsing and validation on the host, the re-layout of every array into the device
// layout of ygg_model.h, one device allocation per model, and the launch entry points.
//
// File format (the reference's, cpu/export.py:34-51,382-468, read by cpu/ygg.cpp:137-220): "YGG1", 11 int32 header
// fields, the array count, a table of (name[32], offset int64, bytes int64), zero padding to 64, the arrays. Beyond
// the reference's limits the loader admits one extension, d_state 96 with readout rank 12 (the readout stored in the
// rank-16 layout with zero rows 12-15); it is laid out on the device as n = 128, R = 16 with zero padding.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <string>
#include <vector>

#include "../../include/ygg_b200.h"
#include "ygg_model.h"

namespace ygg {
cudaError_t launch_step(int n, int blk, int r, int r2p, const DevModel &dm, int B, const int32_t *tok, const int8_t *sin,
                        int8_t *sout, float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int warps,
                        int slots, int grid_cap, cudaStream_t st);
cudaError_t launch_phased(int n, int blk, int r, int r2p, const DevModel &dm, int B, const int32_t *tok,
                          const int8_t *sin, int8_t *sout, float *lg, int32_t *routes, int32_t *acc, int8_t *zq, int warps,
                          int grid_cap, cudaStream_t st);
cudaError_t launch_score(int n, int blk, int r, int r2p, const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state,
                         double *bits, uint32_t rec_max, int warps, int slots, int grid_cap, cudaStream_t st);
size_t block_smem_bytes(uint32_t rec_max, int n, int slots, int warps, int state_bytes);
size_t grouped_ws_bytes(const DevModel &m, int B);
cudaError_t run_grouped(int n, int blk, int r, int r2p, const DevModel &m, int B, int T, const int32_t *tok,
                        int8_t *state, double *bits, void *workspace, int G, int sm_count, cudaStream_t st);
cudaError_t noalloc_scratch(int device, void **ptr, size_t *bytes);
cudaError_t launch_wait_selftest(long long limit, int *d_status, cudaStream_t st);
cudaError_t launch_coop_step(const DevModel &dm, int B, const int32_t *tok, const int8_t *sin, int8_t *sout,
                             float *lg, int32_t *routes, int32_t *acc, uint32_t rec_max, int sm_count, cudaStream_t st);
cudaError_t launch_coop_score(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                              uint32_t rec_max, int sm_count, cudaStream_t st);
cudaError_t launch_pipe_score(const DevModel &dm, int B, int T, const int32_t *tok, int8_t *state, double *bits,
                              uint32_t rec_max, int sm_count, bool split, cudaStream_t st);
}  // namespace ygg

using namespace ygg;

// A launch configuration: the descriptor (device pointers resolved; its records interleaved over lw lanes) and the
// staging slots per block of its step and score kernels.
struct LaunchCfg {
    DevModel dm;
    int slots_step, slots_score;
    bool coop;           // the step / score runs the latency kernels (ygg_coop.cu): 4 warps per stream
    bool phased;         // the step runs layer by layer, one launch per layer (phase_kernel in ygg_step.cu)
    bool pipe;           // the score runs the layer wavefront (ygg_coop.cu): L + 1 groups of 4 warps per row
};

struct ygg_model {
    int device;
    LaunchCfg warp;           // a warp per stream (records over 32 lanes): every shape
    LaunchCfg half;           // two streams per warp (records over 16 lanes), when has_half
    bool has_half;
    // launch policy (ygg_step / ygg_score / grouped, by the batch B): B <= coop_max (n = 128) runs the latency
    // kernels, 4 warps per stream; B <= small_max stages records in shared memory (a warp per stream); B >= big_min
    // runs two streams per warp (fewest instructions per token); in between a warp per stream reads records from
    // global memory. Scoring runs the layer wavefront up to pipe_max rows (n = 128, L <= 7), with a router and an
    // update group per layer when L <= 4 (pipe_split). YGG_COOP (0 or the largest batch), YGG_PIPE (likewise),
    // YGG_PIPE_SPLIT (0 / 1), YGG_LANES (16 / 32) and YGG_DIRECT (0 / 1) fix the choice.
    int coop_max, pipe_max, small_max, big_min, force_lanes, force_direct;
    bool pipe_split;
    uint8_t *d_blob;          // every device array
    size_t d_bytes;
    int *d_status;
    int8_t *d_zq;             // the layer-phased step's readout codes between its launches: [phase_cap][L][32]
    int phase_min, phase_cap; // the step runs layer-phased for phase_min <= B <= phase_cap (direct record reads)
    uint32_t rec_max;
    int warps, grid_cap;
    int sm_count;
    ygg_info_t info;
};

namespace {

#pragma pack(push, 1)
struct FileHeader {
    int32_t n_layers, d_state, block_size, vocab, router_depth, readout_rank, layer_input_rank, reserved,
        router_token_dim, input_rank, shift, n_arrays;
};
struct FileEntry {
    char name[32];
    int64_t offset, bytes;
};
#pragma pack(pop)
static_assert(sizeof(FileHeader) == 48, "YGG1 header");
static_assert(sizeof(FileEntry) == 48, "YGG1 array entry");

struct Arr {
    const uint8_t *p;
    int64_t bytes;
};

size_t round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }

// Host-side plan of the device blob: each array at a 256-byte aligned offset.
struct Blob {
    std::vector<std::pair<size_t, std::vector<uint8_t>>> parts;
    size_t size = 0;
    size_t add(std::vector<uint8_t> &&bytes) {
        const size_t off = size;
        size = round_up(size + bytes.size(), 256);
        parts.emplace_back(off, std::move(bytes));
        return off;
    }
};

// the 16-byte chunk layout: byte `b` of lane `l`'s data in a part interleaved over `lw` lanes
inline size_t lane_byte(int lw, int l, size_t b) { return ((b / 16) * lw + (size_t)l) * 16 + b % 16; }

struct LayerPlan {
    // offsets into the device blob
    size_t rec = 0, rec16 = 0, table = 0, w = 0, thr = 0, vl = 0, mv = 0, mulv = 0, r2b = 0, vt = 0, mt = 0, unembed = 0, sqv = 0;
    bool has_table = false, has_w = false, has_vl = false, has_mulv = false, has_r2b = false, has_vt = false,
         has_sqv = false;
    uint32_t rec_bytes = 0, table_rows = 0;
    uint32_t off_a = kNone, off_u = kNone, off_p = kNone, off_f = kNone, off_cb = kNone, off_su = kNone,
             off_mz = kNone;
    float scal[4] = {0, 0, 0, 0};
};

}  // namespace

extern "C" {

const char *ygg_strerror(int code) {
    switch (code) {
        case YGG_OK: return "ok";
        case YGG_E_ARG: return "bad argument";
        case YGG_E_FORMAT: return "not a YGG1 model file";
        case YGG_E_UNSUPPORTED: return "unsupported model (outside the YGG1 limits)";
        case YGG_E_MISSING: return "missing or malformed model array";
        case YGG_E_CUDA: return "CUDA runtime error";
        case YGG_E_OOM: return "out of memory";
        case YGG_E_TOKEN: return "token out of range";
        case YGG_E_TIMEOUT: return "a bounded device wait gave up";
        case YGG_E_DEVICE: return "no usable sm_100 CUDA device";
        case YGG_E_CAPACITY: return "the batch needs more scratch than the fixed scratch of the allocation-free call holds";
        default: return "unknown error";
    }
}

const char *ygg_version(void) { return "ygg_b200 1.0 sm_100a"; }

int ygg_info(const ygg_model *m, ygg_info_t *out) {
    if (!m || !out) return YGG_E_ARG;
    *out = m->info;
    return YGG_OK;
}

void ygg_free(ygg_model *m) {
    if (!m) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(m->device);
    cudaFree(m->d_blob);
    if (prev >= 0) cudaSetDevice(prev);
    delete m;
}

int ygg_load(const void *file_bytes, size_t nbytes, int device, ygg_model **out) {
    if (!file_bytes || !out) return YGG_E_ARG;
    *out = nullptr;
    const uint8_t *f = (const uint8_t *)file_bytes;
    // ---- header and limits (cpu/ygg.cpp:137-148, cpu/export.py:47-48,353-379)
    if (nbytes < 4 + sizeof(FileHeader) || memcmp(f, "YGG1", 4)) return YGG_E_FORMAT;
    FileHeader h;
    memcpy(&h, f + 4, sizeof h);
    const int L = h.n_layers, nf = h.d_state, b = h.block_size, V = h.vocab, D = h.router_depth, Rf = h.readout_rank,
              R2 = h.layer_input_rank, K = h.input_rank;
    // nf, Rf: the file's state size and readout rank; n, R: the device layout's (the extension pads 96 -> 128 and
    // 12 -> 16); Rs: readout rows as stored in the file (rank 12 takes the rank-16 layout)
    const bool ok = (nf == 64 || nf == 96 || nf == 128 || nf == 256) && (b == 8 || b == 16) &&
                    (Rf == 8 || Rf == 12 || Rf == 16 || Rf == 32) &&
                    R2 >= 0 && R2 <= 64 && R2 % 4 == 0 && L >= 1 && L <= kMaxLayers && V >= 1 && V <= 256 &&
                    D >= 0 && D <= 16 && (L == 1 || D >= 1) && h.reserved == 0 && h.shift >= 1 && h.shift <= 30 &&
                    K >= 0 && K <= 64 && K % 4 == 0;
    if (!ok) return YGG_E_UNSUPPORTED;
    if (h.n_arrays < 0 || nbytes < 4 + sizeof(FileHeader) + (size_t)h.n_arrays * sizeof(FileEntry)) return YGG_E_FORMAT;
    size_t pos = 4 + sizeof(FileHeader) + (size_t)h.n_arrays * sizeof(FileEntry);
    pos = round_up(pos, 64);
    if (pos > nbytes) return YGG_E_FORMAT;
    const size_t avail = nbytes - pos;
    std::map<std::string, Arr> arr;
    for (int i = 0; i < h.n_arrays; i++) {
        FileEntry e;
        memcpy(&e, f + 4 + sizeof(FileHeader) + (size_t)i * sizeof(FileEntry), sizeof e);
        if (e.offset < 0 || e.bytes < 0 || (size_t)e.offset > avail || (size_t)e.bytes > avail - (size_t)e.offset)
            return YGG_E_FORMAT;
        arr[std::string(e.name, strnlen(e.name, 32))] = Arr{f + pos + e.offset, e.bytes};
    }
    const int n = nf == 96 ? 128 : nf, R = Rf == 12 ? 16 : Rf, Rs = Rf == 12 ? 16 : Rf;
    // record layouts: interleaved over 32 lanes (a warp per stream) always, and over 16 lanes (two streams per warp)
    // where a half-warp's share of the work fits its registers (n <= 128 and readout rank <= 16), unless
    // YGG_LANES=32 asks for the warp per stream only
    bool lay16 = n <= 128 && R <= 16;
    if (const char *e = getenv("YGG_LANES")) { if (atoi(e) == 32) lay16 = false; }
    const int E = 1 << D, VP = (V + kClassPad - 1) / kClassPad * kClassPad;
    const int R2P = (int)round_up(R2, 16), KP = (int)round_up(K, 16), NG = n / 16, NGf = nf / 16;
    auto get = [&](int l, const char *tag, int64_t want, Arr &a) -> int {  // 1 found, 0 absent, <0 bad size
        const auto it = arr.find("l" + std::to_string(l) + "_" + tag);
        if (it == arr.end()) return 0;
        if (want >= 0 && it->second.bytes != want) return -1;
        a = it->second;
        return 1;
    };
    const auto hb = arr.find("head_b");
    if (hb == arr.end() || hb->second.bytes != 4 * VP) return YGG_E_MISSING;

    Blob blob;
    LayerPlan plan[kMaxLayers];
    bool any_factored = false, any_group = false, any_mz = false;
    {
        std::vector<uint8_t> ob(4 * (size_t)VP);
        memcpy(ob.data(), hb->second.p, ob.size());
        blob.add(std::move(ob));   // head_b at offset 0
    }
    for (int l = 0; l < L; l++) {
        LayerPlan &P = plan[l];
        const int Ee = l == 0 ? V : E;   // experts of the layer: the token layer has one per token
        Arr meta, rec, Q, scal;
        if (get(l, "meta", -1, meta) != 1 || get(l, "rec", -1, rec) != 1 || get(l, "Q", (int64_t)Rf * VP, Q) != 1 ||
            get(l, "scal", 16, scal) != 1)
            return YGG_E_MISSING;
        if (meta.bytes != 20 && meta.bytes != 32) return YGG_E_MISSING;
        int32_t mt[8] = {0, -1, -1, -1, -1, -1, -1, -1};
        memcpy(mt, meta.p, meta.bytes);
        const int rb = mt[0];
        if (rb <= 0 || rec.bytes != (int64_t)Ee * rb) return YGG_E_MISSING;
        memcpy(P.scal, scal.p, 16);
        Arr vt, mT;
        const int hv = get(l, "vt", (int64_t)V * K, vt);
        if (hv < 0) return YGG_E_MISSING;
        const bool fact = hv == 1;
        if (fact && (K < 4 || meta.bytes != 32 || get(l, "mT", 4 * (int64_t)nf, mT) != 1)) return YGG_E_MISSING;
        const bool low = l > 0 && R2 > 0;
        auto part_ok = [&](int off, int64_t size) { return off >= 0 && (int64_t)off + size <= rb; };
        if (!part_ok(mt[1], 2LL * nf * b) || !part_ok(mt[3], (int64_t)Rs * nf)) return YGG_E_MISSING;
        if (low && !part_ok(mt[2], (int64_t)nf * R2)) return YGG_E_MISSING;
        if (fact) {
            if (!part_ok(mt[5], (int64_t)nf * K) || !part_ok(mt[6], 2LL * nf) || !part_ok(mt[7], 4)) return YGG_E_MISSING;
        } else {
            // table rows: V per routed expert, the own row for the token layer (cpu/ygg.cpp:188)
            if (!part_ok(mt[4], (l == 0 ? 2LL : 2LL * V) * nf)) return YGG_E_MISSING;
        }
        Arr mzl, sqv;
        const int hmz = get(l, "mzl", (int64_t)Ee * (Rf == 8 ? 16 : Rf) * 4, mzl);
        const int hsq = get(l, "sqv", 4LL * VP, sqv);
        if (hmz < 0 || hsq < 0) return YGG_E_MISSING;

        // ---- the device record
        uint32_t off = 0;
        P.off_a = off; off += 2u * n * b;
        if (low) { P.off_u = off; off += (uint32_t)(n * R2P); }
        P.off_p = off; off += (uint32_t)(R * n);
        if (fact) {
            P.off_f = off; off += (uint32_t)(n * KP);
            P.off_cb = off; off += (uint32_t)round_up(2 * n, 16);
            P.off_su = off; off += 16;
        }
        if (hmz == 1) { P.off_mz = off; off += (uint32_t)round_up(4 * R, 16); }
        P.rec_bytes = (uint32_t)round_up(off, 128);
        // the records interleaved over lw lanes (C = n / lw coordinates per lane)
        auto records = [&](const int lw) {
            const int C = n / lw;
            std::vector<uint8_t> dr((size_t)Ee * P.rec_bytes, 0);
            for (int r = 0; r < Ee; r++) {
                const uint8_t *src = rec.p + (size_t)r * rb;
                uint8_t *dst = dr.data() + (size_t)r * P.rec_bytes;
                const int16_t *A = (const int16_t *)(src + mt[1]);
                // transition: lane data word ii * b/2 + p = (A[i][c0 + 2p], A[i][c0 + 2p + 1]); file element (i, jj) of the
                // row's block at ((i/16) * b/2 + jj/2) * 16 + i%16) * 2 + jj%2 (cpu/export.py:321-326)
                uint8_t *pa = dst + P.off_a;
                for (int ln = 0; ln < lw; ln++)
                    for (int ii = 0; ii < C; ii++) {
                        const int i = C * ln + ii;
                        if (i >= nf) continue;   // padded coordinates: zero rows
                        for (int jj = 0; jj < b; jj++) {
                            const int16_t v = A[(((i / 16) * (b / 2) + jj / 2) * 16 + i % 16) * 2 + jj % 2];
                            const size_t lb = (size_t)(ii * (b / 2) + jj / 2) * 4 + (jj % 2) * 2;
                            memcpy(pa + lane_byte(lw, ln, lb), &v, 2);   // lb even: both bytes in one chunk
                        }
                    }
                // projections u8 (u + 128) [rank/4][n][4] (cpu/export.py:329-332) -> lane bytes ii * rankP + k, signed
                auto proj = [&](const uint8_t *u, int rank, int rankp, uint8_t *pd) {
                    for (int ln = 0; ln < lw; ln++)
                        for (int ii = 0; ii < C; ii++) {
                            const int i = C * ln + ii;
                            if (i >= nf) continue;
                            for (int k = 0; k < rank; k++)
                                pd[lane_byte(lw, ln, (size_t)ii * rankp + k)] =
                                    (uint8_t)(u[((size_t)(k / 4) * nf + i) * 4 + k % 4] - 128);
                        }
                };
                if (low) proj(src + mt[2], R2, R2P, dst + P.off_u);
                // readout u8 (p + 128) (cpu/export.py:335-342) -> lane bytes r * C + cc = P[r][C l + cc], signed
                uint8_t *pp = dst + P.off_p;
                const uint8_t *ps = src + mt[3];
                for (int ln = 0; ln < lw; ln++)
                    for (int rr = 0; rr < Rf; rr++)
                        for (int cc = 0; cc < C; cc++) {
                            const int i = C * ln + cc;
                            if (i >= nf) continue;
                            const size_t idx = Rf == 8 ? ((size_t)(i / 8) * 16 + 2 * rr + (i % 8) / 4) * 4 + i % 4
                                                       : ((size_t)((rr / 16) * (nf / 4) + i / 4) * 16 + rr % 16) * 4 + i % 4;
                            pp[lane_byte(lw, ln, (size_t)rr * C + cc)] = (uint8_t)(ps[idx] - 128);
                        }
                if (fact) {
                    proj(src + mt[5], K, KP, dst + P.off_f);
                    memcpy(dst + P.off_cb, src + mt[6], 2 * (size_t)nf);
                    memcpy(dst + P.off_su, src + mt[7], 4);
                }
                if (hmz == 1) {   // R = 8: the file holds each row's scale twice (lanes 2r, 2r+1)
                    const float *mz = (const float *)mzl.p + (size_t)r * (Rf == 8 ? 16 : Rf);
                    for (int rr = 0; rr < Rf; rr++) memcpy(dst + P.off_mz + 4 * rr, mz + (Rf == 8 ? 2 * rr : rr), 4);
                }
            }
            return dr;
        };
        P.rec = blob.add(records(32));
        if (lay16) P.rec16 = blob.add(records(16));
        if (!fact) {   // table rows int16, contiguous per expert
            P.table_rows = l == 0 ? 1 : (uint32_t)V;
            std::vector<uint8_t> t((size_t)Ee * P.table_rows * 2 * n, 0);
            for (int r = 0; r < Ee; r++)
                for (uint32_t row = 0; row < P.table_rows; row++)
                    memcpy(t.data() + ((size_t)r * P.table_rows + row) * 2 * n,
                           rec.p + (size_t)r * rb + mt[4] + (size_t)row * 2 * nf, 2 * (size_t)nf);
            P.table = blob.add(std::move(t));
            P.has_table = true;
        } else {
            std::vector<uint8_t> c((size_t)V * KP, 0);
            for (int x = 0; x < V; x++) memcpy(c.data() + (size_t)x * KP, vt.p + (size_t)x * K, K);
            P.vt = blob.add(std::move(c));
            P.has_vt = true;
            std::vector<uint8_t> ts(4 * (size_t)n, 0);
            memcpy(ts.data(), mT.p, 4 * (size_t)nf);
            P.mt = blob.add(std::move(ts));
            any_factored = true;
        }
        // ---- shared per-layer arrays
        {   // unembedding u8 (q + 128) [R/4][VP][4] (cpu/export.py:345-350) -> s8 [VP][R] (class c = 32 m + lane)
            std::vector<uint8_t> q((size_t)VP * R, 0);
            for (int c = 0; c < VP; c++)
                for (int k = 0; k < Rf; k++) q[(size_t)c * R + k] = (uint8_t)(Q.p[((size_t)(k / 4) * VP + c) * 4 + k % 4] - 128);
            P.unembed = blob.add(std::move(q));
        }
        if (hsq == 1) { P.sqv = blob.add(std::vector<uint8_t>(sqv.p, sqv.p + 4 * VP)); P.has_sqv = true; }
        if (hmz == 1) any_mz = true;
        if (l > 0) {
            Arr w, thr;
            if (get(l, "w", (int64_t)E * nf, w) != 1 || get(l, "thr", 4LL * V * E, thr) != 1) return YGG_E_MISSING;
            std::vector<uint8_t> ws((size_t)E * n, 0);
            for (int e = 0; e < E; e++)   // u8 (w + 128) -> s8 w
                for (int j = 0; j < nf; j++) ws[(size_t)e * n + j] = (uint8_t)(w.p[(size_t)e * nf + j] - 128);
            P.w = blob.add(std::move(ws));
            P.thr = blob.add(std::vector<uint8_t>(thr.p, thr.p + 4 * (size_t)V * E));
            P.has_w = true;
            if (R2) {
                const int RG = R2P / 16;
                Arr vl, mv;
                if (get(l, "vl", (int64_t)RG * 16 * nf, vl) != 1 || get(l, "mv", 4LL * 16 * RG, mv) != 1)
                    return YGG_E_MISSING;
                // u8 (v + 128) [RG][n/4][16][4] (cpu/export.py:402-409) -> s8 [n/16][R2P][16]: lane k's chunk j
                std::vector<uint8_t> d((size_t)NG * R2P * 16, 0);
                for (int k = 0; k < R2P; k++)
                    for (int col = 0; col < nf; col++)
                        d[((size_t)(col / 16) * R2P + k) * 16 + col % 16] =
                            (uint8_t)(vl.p[(((size_t)(k / 16) * (nf / 4) + col / 4) * 16 + k % 16) * 4 + col % 4] - 128);
                P.vl = blob.add(std::move(d));
                P.mv = blob.add(std::vector<uint8_t>(mv.p, mv.p + 4 * R2P));
                P.has_vl = true;
            }
            Arr mulv, r2b;
            const int hm = get(l, "mulv", 4LL * nf, mulv), hr = get(l, "r2b", 4LL * NGf, r2b);
            if (hm < 0 || hr < 0) return YGG_E_MISSING;
            auto padded = [](const Arr &a, size_t bytes) {   // a's bytes, zero padded to `bytes`
                std::vector<uint8_t> v(bytes, 0);
                memcpy(v.data(), a.p, (size_t)a.bytes);
                return v;
            };
            if (hm == 1) { P.mulv = blob.add(padded(mulv, 4 * (size_t)n)); P.has_mulv = true; }
            if (hr == 1) { P.r2b = blob.add(padded(r2b, 4 * (size_t)NG)); P.has_r2b = true; any_group = true; }
        }
    }

    // ---- device
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return YGG_E_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) return YGG_E_DEVICE;
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return YGG_E_DEVICE;
    ygg_model *m = new ygg_model();
    m->device = device;
    m->sm_count = prop.multiProcessorCount;
    const size_t status_off = blob.size;
    // the layer-phased step keeps each stream's readout codes (32 bytes a layer) between its launches, in the model's
    // own allocation: up to phase_cap streams a launch
    m->phase_cap = 1 << 18;
    const size_t zq_off = status_off + 256;
    m->d_bytes = zq_off + (size_t)m->phase_cap * L * 32;
    int rc = YGG_OK;
    if (cudaMalloc((void **)&m->d_blob, m->d_bytes) != cudaSuccess) {
        rc = YGG_E_OOM;
    } else {
        for (auto &p : blob.parts)
            if (cudaMemcpy(m->d_blob + p.first, p.second.data(), p.second.size(), cudaMemcpyHostToDevice) != cudaSuccess)
                rc = YGG_E_CUDA;
    }
    if (rc == YGG_OK && cudaMemset(m->d_blob + status_off, 0, 256) != cudaSuccess) rc = YGG_E_CUDA;
    if (rc != YGG_OK) {
        cudaFree(m->d_blob);
        delete m;
        if (prev >= 0) cudaSetDevice(prev);
        return rc;
    }
    uint8_t *d = m->d_blob;
    DevModel &dm = m->warp.dm;
    memset(&dm, 0, sizeof dm);
    dm.L = L; dm.n = n; dm.b = b; dm.V = V; dm.VP = VP; dm.D = D; dm.E = E; dm.R = R; dm.R2 = R2; dm.R2P = R2P;
    dm.K = K; dm.KP = KP; dm.shift = h.shift; dm.factored = any_factored; dm.has_mz = any_mz;
    dm.ns = nf;
    dm.lw = 32;
    dm.direct = 0;                 // set per launch
    dm.inv_n = 1.0f / (float)nf;   // the reference's (1.0f / N) (cpu/ygg.cpp:253), f32(1.0 / n) in int_forward
    dm.head_b = (const float *)d;
    dm.status = (int *)(d + status_off);
    m->d_status = dm.status;
    m->d_zq = (int8_t *)(d + zq_off);
    uint32_t rec_max = 0;
    for (int l = 0; l < L; l++) {
        const LayerPlan &P = plan[l];
        DevLayer &y = dm.layer[l];
        y.rec = d + P.rec; y.rec_bytes = P.rec_bytes;
        y.off_a = P.off_a; y.off_u = P.off_u; y.off_p = P.off_p; y.off_f = P.off_f; y.off_cb = P.off_cb;
        y.off_su = P.off_su; y.off_mz = P.off_mz;
        y.table = P.has_table ? (const int16_t *)(d + P.table) : nullptr;
        y.table_rows = P.table_rows;
        y.w = P.has_w ? (const int8_t *)(d + P.w) : nullptr;
        y.thr = P.has_w ? (const float *)(d + P.thr) : nullptr;
        y.vl = P.has_vl ? (const int8_t *)(d + P.vl) : nullptr;
        y.mv = P.has_vl ? (const float *)(d + P.mv) : nullptr;
        y.mulv = P.has_mulv ? (const float *)(d + P.mulv) : nullptr;
        y.r2b = P.has_r2b ? (const float *)(d + P.r2b) : nullptr;
        y.vt = P.has_vt ? (const int8_t *)(d + P.vt) : nullptr;
        y.mt = P.has_vt ? (const float *)(d + P.mt) : nullptr;
        y.unembed = (const int8_t *)(d + P.unembed);
        y.sqv = P.has_sqv ? (const float *)(d + P.sqv) : nullptr;
        y.readout_scale = P.scal[0]; y.unembed_scale = P.scal[1]; y.rms_eps = P.scal[2]; y.layer_input_scale = P.scal[3];
        if (P.rec_bytes > rec_max) rec_max = P.rec_bytes;
    }
    // the same model with its records interleaved over 16 lanes
    m->has_half = lay16;
    m->half.dm = dm;
    m->half.dm.lw = 16;
    if (lay16)
        for (int l = 0; l < L; l++) m->half.dm.layer[l].rec = d + plan[l].rec16;
    m->rec_max = rec_max;
    // launch shape: W warps per block, each serving 32 / lw streams, share S leaf slots (a stream holds a slot only
    // from its copy to its readout); S is the most slots that still let `blocks` blocks share an SM's shared memory
    const size_t sm_smem = prop.sharedMemPerMultiprocessor, cap = prop.sharedMemPerBlockOptin;
    int W = 8, blocks = n >= 256 ? 2 : 4;   // the kernels' launch bounds (blocks_per_sm in ygg_step.cu)
    if (const char *e = getenv("YGG_WARPS")) { const int v = atoi(e); if (v >= 1 && v <= 8) W = v; }
    if (const char *e = getenv("YGG_BLOCKS_PER_SM")) { const int v = atoi(e); if (v >= 1 && v <= 8) blocks = v; }
    m->warps = W;
    // slots come in units of P = 32 / lw (a warp claims one slot per stream it serves, all at once)
    auto pick_slots = [&](LaunchCfg &c) {
        const int P = 32 / c.dm.lw, streams = W * P;
        auto fit = [&](int state_bytes) {
            int S = streams;
            while (S > P && (block_smem_bytes(rec_max, n, S, streams, state_bytes) + 1024) * blocks > sm_smem) S -= P;
            while (S > P && block_smem_bytes(rec_max, n, S, streams, state_bytes) > cap) S -= P;
            return S;
        };
        // half the streams' worth of slots is plenty (a stream holds one for a small part of a layer) and leaves
        // more of the SM's unified L1/shared memory to the L1 cache
        c.slots_step = std::min(fit(0), (streams / 2 + P - 1) / P * P);
        if (const char *e = getenv("YGG_SLOTS")) {
            const int v = atoi(e) / P * P;
            if (v >= P && v <= streams && block_smem_bytes(rec_max, n, v, streams, 0) <= cap) c.slots_step = v;
        }
        c.slots_score = fit((int)round_up((size_t)L * n, 128));
    };
    pick_slots(m->warp);
    if (lay16) pick_slots(m->half);
    // staging pays below ~2 K streams for n >= 128 (a 10 KB record lands with one bulk copy instead of ~40 loads per
    // lane with few in flight); the smaller records of n = 64 read as fast directly at every batch
    m->small_max = n >= 128 ? 2048 : 0;
    // the latency kernels win up to ~256 streams (c3 step: 14.2 against 16.5 us at 16 streams, 16.6 against 18.3 at
    // 256; c5 score rows: +18 % at 256); from ~512 the warp-per-stream kernels fill the GPU better
    m->coop_max = n == 128 ? 256 : 0;
    // scoring rows: the layer wavefront (one row per SM at a time, ~54 M tokens/s on c3 at any count of rows) wins up
    // to about four rows per SM (592 rows: 53.5 against 45.4 M tokens/s), the other kernels from there (888 rows:
    // 68.3 against 53.8 M)
    m->pipe_max = n == 128 && L <= 7 ? 4 * m->sm_count : 0;
    // two streams per warp from 8 192 streams at n = 128 (c3: 184.5 against 164.3 M tokens/s at 8 192, 208.3 against
    // 187.6 at 16 384; c4: 160.2 against 153.6 at 8 192; at 4 096 a warp per stream wins, 141.6 against 128.5)
    m->big_min = n == 128 ? 8192 : 32768;
    m->force_lanes = 0;
    m->force_direct = -1;
    if (const char *e = getenv("YGG_SMALL_BATCH")) m->small_max = atoi(e);
    if (const char *e = getenv("YGG_COOP")) m->coop_max = n == 128 ? atoi(e) : 0;
    m->phase_min = 1 << 30;
    if (const char *e = getenv("YGG_PHASED")) m->phase_min = atoi(e) > 0 ? atoi(e) : 1 << 30;
    if (const char *e = getenv("YGG_PIPE")) m->pipe_max = n == 128 && L <= 7 ? atoi(e) : 0;
    m->pipe_split = true;
    if (const char *e = getenv("YGG_PIPE_SPLIT")) m->pipe_split = atoi(e) != 0;
    if (const char *e = getenv("YGG_BIG_BATCH")) m->big_min = atoi(e);
    if (const char *e = getenv("YGG_LANES")) m->force_lanes = atoi(e) == 16 ? 16 : atoi(e) == 32 ? 32 : 0;
    if (const char *e = getenv("YGG_DIRECT")) m->force_direct = atoi(e) != 0;
    m->grid_cap = 1 << 30;
    ygg_info_t &inf = m->info;
    memset(&inf, 0, sizeof inf);
    inf.n_layers = L; inf.d_state = nf; inf.block_size = b; inf.vocab = V; inf.router_depth = D; inf.readout_rank = Rf;
    inf.layer_input_rank = R2; inf.router_token_dim = h.router_token_dim; inf.input_rank = K; inf.shift = h.shift;
    inf.n_experts = E; inf.vocab_pad = VP; inf.factored = any_factored; inf.group_scales = any_group;
    inf.file_array_bytes = (int64_t)avail; inf.device_bytes = (int64_t)m->d_bytes; inf.record_bytes = (int32_t)rec_max;
    inf.warps_per_block = m->warps;
    inf.slots_per_block = m->warp.slots_step;
    if (prev >= 0) cudaSetDevice(prev);
    *out = m;
    return YGG_OK;
}

// The configuration a launch over `batch` streams (or rows) runs with, its record path set (the launch policy of
// ygg_model).
static LaunchCfg choose(const ygg_model *m, int batch) {
    const bool half = m->has_half && (m->force_lanes == 16 || (m->force_lanes == 0 && batch >= m->big_min));
    LaunchCfg c = half ? m->half : m->warp;
    c.dm.direct = m->force_direct >= 0 ? m->force_direct : (batch > m->small_max ? 1 : 0);
    c.coop = !half && m->force_lanes == 0 && m->force_direct < 0 && batch <= m->coop_max;
    c.pipe = !half && m->force_lanes == 0 && m->force_direct < 0 && batch <= m->pipe_max;
    c.phased = c.dm.direct && !c.coop && batch >= m->phase_min && batch <= m->phase_cap;
    return c;
}

static int set_device(const ygg_model *m, int *prev) {
    *prev = -1;
    cudaGetDevice(prev);
    if (*prev != m->device && cudaSetDevice(m->device) != cudaSuccess) return YGG_E_CUDA;
    return YGG_OK;
}
static void restore_device(const ygg_model *m, int prev) {
    if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
}

int ygg_step_debug(const ygg_model *m, int batch, const int32_t *d_tokens, const int8_t *d_state_in,
                   int8_t *d_state_out, float *d_logits, int32_t *d_routes, int32_t *d_acc, void *stream) {
    if (!m || batch < 0) return YGG_E_ARG;
    if (batch == 0) return YGG_OK;
    if (!d_tokens || !d_state_in || !d_state_out) return YGG_E_ARG;
    int prev;
    if (set_device(m, &prev)) return YGG_E_CUDA;
    const LaunchCfg c = choose(m, batch);
    const DevModel &dm = c.dm;
    const cudaError_t e =
        c.coop ? launch_coop_step(dm, batch, d_tokens, d_state_in, d_state_out, d_logits, d_routes, d_acc, m->rec_max,
                                  m->sm_count, (cudaStream_t)stream)
        : c.phased ? launch_phased(dm.n, dm.b, dm.R, dm.R2P, dm, batch, d_tokens, d_state_in, d_state_out, d_logits,
                                   d_routes, d_acc, m->d_zq, m->warps, m->grid_cap, (cudaStream_t)stream)
                   : launch_step(dm.n, dm.b, dm.R, dm.R2P, dm, batch, d_tokens, d_state_in, d_state_out, d_logits, d_routes,
                                 d_acc, m->rec_max, m->warps, c.slots_step, m->grid_cap, (cudaStream_t)stream);
    restore_device(m, prev);
    return e == cudaSuccess ? YGG_OK : YGG_E_CUDA;
}

int ygg_step(const ygg_model *m, int batch, const int32_t *d_tokens, const int8_t *d_state_in, int8_t *d_state_out,
             float *d_logits, void *stream) {
    return ygg_step_debug(m, batch, d_tokens, d_state_in, d_state_out, d_logits, nullptr, nullptr, stream);
}

int ygg_score(const ygg_model *m, int batch, int steps, const int32_t *d_tokens, int8_t *d_state, double *d_bits,
              void *stream) {
    if (!m || batch < 0 || steps < 0) return YGG_E_ARG;
    if (batch == 0) return YGG_OK;
    if (!d_tokens || !d_bits) return YGG_E_ARG;
    int prev;
    if (set_device(m, &prev)) return YGG_E_CUDA;
    const LaunchCfg c = choose(m, batch);
    const DevModel &dm = c.dm;
    const cudaError_t e =
        c.pipe   ? launch_pipe_score(dm, batch, steps, d_tokens, d_state, d_bits, m->rec_max, m->sm_count,
                                     m->pipe_split, (cudaStream_t)stream)
        : c.coop ? launch_coop_score(dm, batch, steps, d_tokens, d_state, d_bits, m->rec_max, m->sm_count,
                                     (cudaStream_t)stream)
                 : launch_score(dm.n, dm.b, dm.R, dm.R2P, dm, batch, steps, d_tokens, d_state, d_bits, m->rec_max,
                              m->warps, c.slots_score, m->grid_cap, (cudaStream_t)stream);
    restore_device(m, prev);
    return e == cudaSuccess ? YGG_OK : YGG_E_CUDA;
}

size_t ygg_score_grouped_workspace(const ygg_model *m, int batch) {
    if (!m || batch < 0) return 0;
    return grouped_ws_bytes(m->warp.dm, batch);
}

int ygg_score_grouped(const ygg_model *m, int batch, int steps, const int32_t *d_tokens, int8_t *d_state,
                      double *d_bits, int min_group, void *d_workspace, size_t workspace_bytes, void *stream) {
    if (!m || batch < 0 || steps < 0) return YGG_E_ARG;
    if (batch == 0) return YGG_OK;
    if (!d_tokens || !d_bits || !d_workspace || ((uintptr_t)d_workspace & 255) ||
        workspace_bytes < grouped_ws_bytes(m->warp.dm, batch))
        return YGG_E_ARG;
    int prev;
    if (set_device(m, &prev)) return YGG_E_CUDA;
    const LaunchCfg c = choose(m, batch);
    const DevModel &dm = c.dm;
    const cudaError_t e = run_grouped(dm.n, dm.b, dm.R, dm.R2P, dm, batch, steps, d_tokens,
                                      d_state, d_bits, d_workspace, min_group, m->sm_count, (cudaStream_t)stream);
    restore_device(m, prev);
    return e == cudaSuccess ? YGG_OK : YGG_E_CUDA;
}

int ygg_score_grouped_noalloc(const ygg_model *m, int batch, int steps, const int32_t *d_tokens, int8_t *d_state,
                              double *d_bits, int min_group, void *stream) {
    if (!m || batch < 0 || steps < 0) return YGG_E_ARG;
    if (batch == 0) return YGG_OK;
    if (!d_tokens || !d_bits) return YGG_E_ARG;
    const size_t need = grouped_ws_bytes(m->warp.dm, batch);
    int prev;
    if (set_device(m, &prev)) return YGG_E_CUDA;
    void *scratch = nullptr;
    size_t cap = 0;
    if (noalloc_scratch(m->device, &scratch, &cap) != cudaSuccess) {
        restore_device(m, prev);
        return YGG_E_CUDA;
    }
    if (need > cap) {
        restore_device(m, prev);
        return YGG_E_CAPACITY;
    }
    const LaunchCfg c = choose(m, batch);
    const DevModel &dm = c.dm;
    const cudaError_t e = run_grouped(dm.n, dm.b, dm.R, dm.R2P, dm, batch, steps, d_tokens,
                                      d_state, d_bits, scratch, min_group, m->sm_count, (cudaStream_t)stream);
    restore_device(m, prev);
    return e == cudaSuccess ? YGG_OK : YGG_E_CUDA;
}

int ygg_selftest_wait(int device, long long cycles, void *stream, int *status_out) {
    if (!status_out || cycles < 0) return YGG_E_ARG;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return YGG_E_DEVICE;
    int prev = -1;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return YGG_E_DEVICE;
    int *d = nullptr, v = -1;
    cudaError_t e = cudaMalloc((void **)&d, sizeof(int));
    if (e == cudaSuccess) e = launch_wait_selftest(cycles, d, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&v, d, sizeof v, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    cudaFree(d);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess) return YGG_E_CUDA;
    *status_out = (v & kStatusTimeout) ? YGG_E_TIMEOUT : YGG_OK;
    return YGG_OK;
}

int ygg_status(const ygg_model *m, void *stream, int clear, int *status_out) {
    if (!m || !status_out) return YGG_E_ARG;
    int prev;
    if (set_device(m, &prev)) return YGG_E_CUDA;
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, m->d_status, sizeof v, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e == cudaSuccess && clear) {
        e = cudaMemsetAsync(m->d_status, 0, sizeof(int), (cudaStream_t)stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    }
    restore_device(m, prev);
    if (e != cudaSuccess) return YGG_E_CUDA;
    *status_out = (v & kStatusTimeout) ? YGG_E_TIMEOUT : (v & kStatusBadToken) ? YGG_E_TOKEN : YGG_OK;
    return YGG_OK;
}

}  // extern "C"
