// Device layout of a loaded model, shared by the loader (ygg_load.cu) and the kernels (ygg_step.cu).
//
// A stream is served by LW lanes (lw: 32, a warp, or 16, half a warp; the loader picks 16 for n = 64 / 128 with
// readout rank <= 16). Lane l of the group owns the C = n/LW state coordinates [C l, C l + C) of every layer, and
// every per-expert array is re-laid out at load time so that the bytes lane l needs sit in the lane's own 16-byte
// chunks: chunk j of lane l is at byte (LW j + l) * 16 of the part. One 16-byte load of the group therefore reads
// 16 LW contiguous bytes (conflict-free in shared memory, fully coalesced in global memory), and a whole expert
// record is one contiguous block that a single bulk copy (cp.async.bulk) brings into the stream's shared-memory slot.
//
// Per-expert record (rec_bytes each, a multiple of 128):
//   A   transition int16, lane data = C rows x BLK columns of the row's own diagonal block, as (C * BLK / 2) words
//       word ii * BLK/2 + p = (A[i][c0 + 2p], A[i][c0 + 2p + 1]), i = C l + ii, c0 = (i / BLK) * BLK
//   U'  layer-input projection int8 (routed layers with R2 > 0): C rows x R2P columns (zero padded)
//   P   readout int8: C >= 4: word r * C/4 + w = P[r][C l + 4w .. +3]; C = 2: word w = (P[2w][2l..], P[2w+1][2l..])
//   F   factored input projection int8: C rows x KP columns (zero padded)
//   CB  factored bias c_r int16 [n] (plain layout), SU: su_r f32 (16-byte slot)
//   MZ  group readout scales f32 [R] (per expert and readout row)
// Shared per layer: router rows s8 [E][n] (heap order, row 0 unused), thresholds f32 [V][E], the layer-input down
// projection s8 [n/16][R2P][16] (lane k reads its row k as 16-byte chunks), mv f32 [R2P], tables int16 rows of n,
// token codes s8 [V][KP], the unembedding s8 [VP/32][32][R] (class 32 m + lane), optional group scales.
//
// A file of the d_state 96 extension (readout rank 12) is laid out as n = 128 and R = 16 with zero rows and columns:
// the padded coordinates see zero weights everywhere, so they stay 0 and add nothing to any dot, and the kernels run
// the n = 128 code. Only two things keep the file's n: the caller's state layout (ns coordinates per layer) and rho's
// f32(1 / ns).
#pragma once
#include <stdint.h>

namespace ygg {

constexpr int kMaxLayers = 8;
constexpr int kClassPad = 32;
constexpr uint32_t kNone = 0xFFFFFFFFu;
constexpr int kWaitLimitCycles = 1 << 31;   // bounded device waits: ~1 s at 1.9 GHz, then an error status

enum Status : int {
    kStatusOk = 0,
    kStatusBadToken = 1,
    kStatusTimeout = 2,
};

struct DevLayer {
    const uint8_t *rec;          // E records (the token layer: V records, expert = token)
    uint32_t rec_bytes;          // bytes per record, multiple of 128
    uint32_t off_a, off_u, off_p, off_f, off_cb, off_su, off_mz;   // byte offsets in the record, kNone: absent
    const int16_t *table;        // table rows, or null (factored)
    uint32_t table_rows;         // rows per expert: V (routed) or 1 (token layer: row of expert x)
    const int8_t *w;             // router rows s8 [E][n]
    const float *thr;            // thresholds [V][E]
    const int8_t *vl;            // down projection s8 [n/16][R2P][16]
    const float *mv;             // [R2P]
    const float *mulv;           // [n] per-coordinate layer-input scale, or null
    const float *r2b;            // [n/16] squared relative group scales of the layer below, or null
    const int8_t *vt;            // factored token codes s8 [V][KP], or null
    const float *mt;             // factored token scale [n], or null
    const int8_t *unembed;       // s8 [VP/32][32][R]
    const float *sqv;            // per-class unembedding scale [VP], or null
    float readout_scale, unembed_scale, rms_eps, layer_input_scale;
};

struct DevModel {
    int L, n, b, V, VP, D, E, R, R2, R2P, K, KP, shift;   // n, R: the device layout's (padded) sizes
    int lw;                      // lanes per stream of the record layout and the kernels: 32 or 16
    int direct;                  // 1: the fast step / score kernels read records from global memory (no staging)
    int ns;                      // state coordinates per layer in the caller's layout: the file's d_state (<= n)
    float inv_n;                 // f32(1 / ns), rho's mean factor
    int factored, has_mz;
    const float *head_b;         // [VP]
    int *status;                 // device status word (bit flags of Status)
    DevLayer layer[kMaxLayers];
};

}  // namespace ygg
