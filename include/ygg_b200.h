/* ygg_b200: the int8 streaming inference step of Yggdrasil on NVIDIA B200 (sm_100a), as a C-ABI library.
 *
 * Plain pointers and sizes only: device pointers are raw CUDA device addresses (for example torch.Tensor.data_ptr()
 * of a CUDA tensor), `stream` is a cudaStream_t passed as void* (NULL: the legacy default stream). Every compute
 * call is asynchronous on that stream; the model handle is read-only after ygg_load, so calls on different streams
 * may share it. One handle serves one device.
 *
 * Errors: 0 = YGG_OK, a negative YGG_E_* code otherwise (ygg_strerror). No call exits the process, unlike the
 * reference's die() (cpu/ygg.cpp:41-43).
 *
 * Each entry point names the reference interface it replaces, by file:line in the reference repository.
 */
#ifndef YGG_B200_H
#define YGG_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define YGG_API __attribute__((visibility("default")))
#else
#define YGG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define YGG_OK 0
#define YGG_E_ARG (-1)          /* bad argument: null pointer, negative size */
#define YGG_E_FORMAT (-2)       /* not a YGG1 file, or its array table does not fit the file */
#define YGG_E_UNSUPPORTED (-3)  /* header outside the format limits (cpu/export.py:47-48, cpu/ygg.cpp:141-146) and
                                   the d_state 96 extension (ygg_load) */
#define YGG_E_MISSING (-4)      /* a required array is absent or has the wrong size */
#define YGG_E_CUDA (-5)         /* a CUDA runtime call failed */
#define YGG_E_OOM (-6)          /* device or host allocation failed */
#define YGG_E_TOKEN (-7)        /* a token outside [0, vocab) (cpu/ygg.cpp:493-495) */
#define YGG_E_TIMEOUT (-8)      /* a bounded device wait gave up (reported through ygg_status) */
#define YGG_E_DEVICE (-9)       /* no such CUDA device, or not an sm_100 device */
#define YGG_E_CAPACITY (-10)    /* the batch needs more scratch than ygg_score_grouped_noalloc's fixed scratch holds */

typedef struct ygg_model ygg_model;

/* Shape of a loaded model: the YGG1 header fields (cpu/export.py:41-42, cpu/ygg.cpp:79-82) plus derived sizes. */
typedef struct {
    int32_t n_layers, d_state, block_size, vocab, router_depth, readout_rank, layer_input_rank, router_token_dim,
        input_rank, shift;
    int32_t n_experts;          /* 2^router_depth */
    int32_t vocab_pad;          /* vocab rounded up to 32 */
    int32_t factored;           /* 1: routed layers store U_r, c_r (factored input), 0: tables T_r[x] */
    int32_t group_scales;       /* 1: per-group state scales (r2b) are present */
    int64_t file_array_bytes;   /* bytes of the file's array section */
    int64_t device_bytes;       /* bytes the handle holds on the device */
    int32_t record_bytes;       /* largest per-expert record in the device layout */
    int32_t warps_per_block;    /* launch shape of the step kernel: warps per block ... */
    int32_t slots_per_block;    /* ... sharing this many shared-memory leaf slots */
} ygg_info_t;

/* Parse a YGG1 file held in host memory, re-lay it out for the device and upload it to `device`.
 * Replaces the reference loader: cpu/ygg.cpp:204-220 (load), :137-148 (read_header), :151-171 (read_blob),
 * :173-202 (bind_layer); the file format is cpu/export.py:34-51,382-468. Beyond the reference's limits it also
 * admits d_state 96 with readout rank 12 (that readout stored in the rank-16 layout with zero rows 12-15), a format
 * extension of this library; ygg_info then reports d_state 96, and every state buffer is [..][n_layers][96]. */
YGG_API int ygg_load(const void *file_bytes, size_t nbytes, int device, ygg_model **out);

/* Shape and sizes of a loaded model. */
YGG_API int ygg_info(const ygg_model *m, ygg_info_t *out);

/* One decode step of `batch` independent streams: for every layer the router descent, the leaf gather, the
 * transition / input / layer-input update with saturation, and the readout into the logits.
 *   d_tokens     int32 [batch]
 *   d_state_in   int8  [batch][n_layers][d_state]   (may equal d_state_out: updated in place)
 *   d_state_out  int8  [batch][n_layers][d_state]
 *   d_logits     float [batch][vocab]   or NULL (logits not written)
 * Replaces cpu/ygg.cpp:441-459 (step, one stream) and the step of yggdrasil/inference.py:175-177 /
 * yggdrasil/inference_triton.py:187-212 (B streams per launch). */
YGG_API int ygg_step(const ygg_model *m, int batch, const int32_t *d_tokens, const int8_t *d_state_in, int8_t *d_state_out,
             float *d_logits, void *stream);

/* ygg_step that also writes what the reference kernel keeps internal, for bit-exact checks:
 *   d_routes  int32 [batch][n_layers]           the leaf (expert) of each layer; the token for layer 0; or NULL
 *   d_acc     int32 [batch][n_layers][d_state]  the int32 accumulator before saturation to int8; or NULL
 * Same arithmetic as ygg_step (cpu/ygg.cpp:271-280 route, :380-389 update). */
YGG_API int ygg_step_debug(const ygg_model *m, int batch, const int32_t *d_tokens, const int8_t *d_state_in,
                   int8_t *d_state_out, float *d_logits, int32_t *d_routes, int32_t *d_acc, void *stream);

/* Score `batch` rows of `steps` tokens in one launch, state and logits kept on chip:
 *   d_bits[b] = sum over t < steps-1 of -log2 softmax(logits after token t)[token t+1], in float64
 *   d_tokens  int32 [batch][steps]
 *   d_state   int8  [batch][n_layers][d_state] in/out (the state after the first steps-1 tokens), or NULL: zero
 * Replaces yggdrasil/inference.py:179-188 / inference_triton.py:214-227 (score) with the float64 NLL of
 * cpu/ygg.cpp:513-517. */
YGG_API int ygg_score(const ygg_model *m, int batch, int steps, const int32_t *d_tokens, int8_t *d_state, double *d_bits,
              void *stream);

/* Bytes of device workspace ygg_score_grouped needs for `batch` rows. */
YGG_API size_t ygg_score_grouped_workspace(const ygg_model *m, int batch);

/* ygg_score computed step by step with the streams of each layer bucketed by leaf: a leaf that at least `min_group`
 * streams share runs its update as int8 tensor-core GEMMs (tcgen05, n <= 128), the others the per-stream update.
 * Same arguments and bit-identical results as ygg_score; d_workspace: ygg_score_grouped_workspace(m, batch) bytes of
 * device memory owned by the caller (256-byte aligned). The grouping is new: the reference has no counterpart; its
 * result is defined by yggdrasil/inference.py:179-188 and cpu/ygg.cpp:441-459,513-517 as for ygg_score. */
YGG_API int ygg_score_grouped(const ygg_model *m, int batch, int steps, const int32_t *d_tokens, int8_t *d_state,
                              double *d_bits, int min_group, void *d_workspace, size_t workspace_bytes, void *stream);

/* ygg_score_grouped for callers that cannot allocate device memory while they run: a host whose own pool owns the
 * GPU's memory, a serving loop that forbids allocation on its hot path, or a binding with no CUDA allocator. It
 * takes no workspace: its scratch is one fixed 16 MiB array in device memory that every GPU loading this library holds
 * until the process exits, so it calls no allocator at all. A batch whose scratch (ygg_score_grouped_workspace)
 * exceeds 16 MiB is refused with YGG_E_CAPACITY (22 738 rows at n = 128, L = 4, 8192 leaves). The first call on a device
 * looks up the array's device address (once per device and context: after the device's primary context is reset, or
 * under another context, the next call looks it up again); make that first call before any stream capture. Every call
 * shares the array and clears what must start at zero; calls whose work overlaps on the GPU (other streams, other
 * threads) race on it, so run them one after another. Same arguments (less the workspace) and the same results as
 * ygg_score_grouped. No counterpart in the reference: it is an addition of this library. */
YGG_API int ygg_score_grouped_noalloc(const ygg_model *m, int batch, int steps, const int32_t *d_tokens,
                                      int8_t *d_state, double *d_bits, int min_group, void *stream);

/* Read (and with clear != 0, reset) the model's device status word after the calls queued on `stream`:
 * 0 when every call since the last clear ran clean, else a negative YGG_E_* code (token out of range, or a bounded
 * wait that gave up). Synchronises `stream`. */
YGG_API int ygg_status(const ygg_model *m, void *stream, int clear, int *status_out);

/* Self test of the bounded device waits, for failure-detection tests: one warp on `device` waits on an mbarrier that
 * nothing completes, gives up after `cycles` clock cycles exactly as a wait of the step kernels does after ~1 s, and
 * *status_out receives YGG_E_TIMEOUT (YGG_OK had the wait ended). Synchronises `stream`; the context stays usable. No
 * counterpart in the reference (its CPU kernel has no device waits). */
YGG_API int ygg_selftest_wait(int device, long long cycles, void *stream, int *status_out);

/* ---- the fp32 float step (backend "b200f") ------------------------------------------------------------------------
 * The reference's float inference model: yggdrasil/inference.py:42-75 (route, update, step) as its Triton backend
 * fuses it (yggdrasil/inference_triton.py:21-106 and the torch.addmm head, :187-194). Weights are float32 arrays in
 * the checkpoint's own shapes, with the tables T_r[x] = U_r v(x) + c_r and the transitions
 * A_r = diag(clip(decay, -1, 1)) blockdiag(expm((G - G^T) / 2)) already formed (inference_triton.py:109-120). */
typedef struct ygg_fmodel ygg_fmodel;

typedef struct {
    int32_t n_layers, d_state, block_size, vocab, classes, router_depth, router_token_dim, readout_rank,
        layer_input_rank;
    int32_t route_on_state;      /* 1: the router reads [router_embed(x); rms(h_below)] (router_input token_state), 0:
                                    the token part only (router_input token) */
    int32_t token_transition;    /* 1: the token layer has transitions A_x */
    int32_t routed_transition;   /* 1: the routed layers have transitions A_r (expert_type transition) */
} ygg_fshape_t;

/* Host arrays of ygg_fload: YGG_F_ARRAYS_PER_LAYER pointers per layer l, at arrays[l * YGG_F_ARRAYS_PER_LAYER + k],
 * then the output bias (classes) at arrays[n_layers * YGG_F_ARRAYS_PER_LAYER]. E = 2^router_depth, F =
 * router_token_dim, FIN = F + d_state (route_on_state) or F:
 *   k = 0 table: token layer [vocab][d_state] (T_x[x], its own rows); routed [E][vocab][d_state]
 *   k = 1 transition [experts][d_state / block][block][block], or NULL without transitions
 *   k = 2 readout [experts][readout_rank][d_state]      k = 3 unembed [classes][readout_rank]
 *   routed layers only: k = 4 router_embed [vocab][F], k = 5 router_weight [E - 1][FIN], k = 6 router_bias [E - 1],
 *   k = 7 layer_input_down [layer_input_rank][d_state] and k = 8 layer_input_proj [E][d_state][layer_input_rank]
 *   (both NULL when layer_input_rank is 0); k = 4..8 of the token layer are ignored.
 * Limits: d_state 64 / 128 / 256, an even block size <= 32, readout rank <= 32, layer-input rank <= d_state,
 * router_token_dim <= d_state, depth <= 20, 2..16 layers. Replaces TritonYggdrasil.__init__
 * (yggdrasil/inference_triton.py:123-151): the library copies the arrays into its own device layout. */
#define YGG_F_ARRAYS_PER_LAYER 9
YGG_API int ygg_fload(const ygg_fshape_t *shape, const float *const *arrays, int device, ygg_fmodel **out);

/* One fp32 step of `batch` streams (yggdrasil/inference.py:66-75, inference_triton.py:187-194):
 *   d_tokens    int32 [batch]
 *   d_state_in  float [batch][n_layers][d_state]   (may equal d_state_out)
 *   d_state_out float [batch][n_layers][d_state]
 *   d_logits    float [batch][classes]
 *   d_experts   int32 [batch][n_layers] the expert of every layer (the token for the token layer), or NULL
 * A token outside [0, vocab) skips its stream (NaN logits, state copied through) and is reported by ygg_fstatus. */
YGG_API int ygg_fstep(const ygg_fmodel *m, int batch, const int32_t *d_tokens, const float *d_state_in,
                      float *d_state_out, float *d_logits, int32_t *d_experts, void *stream);

/* ygg_fstep that also accumulates the calibration maxima of the reference's exporter (cpu/export.py:120-153,
 * `LayerStats` and `calibrate`: |h| per group of 16 coordinates, |V' rms(h_below)|, |P_r h| per readout row) over the
 * batch, into d_stats: float [n_layers][d_state / 16 + 1 + readout_rank], per layer the group maxima, the layer-input
 * maximum (0 for the token layer) and the row maxima. Each value is the running maximum across every call that passes
 * the same buffer (zero it first); a calibration is a loop of these calls over the steps of its windows. Replaces the
 * JAX scan of `calibrate` (cpu/export.py:129-153) with the fp32 step on the GPU. */
YGG_API int ygg_fstep_stats(const ygg_fmodel *m, int batch, const int32_t *d_tokens, const float *d_state_in,
                            float *d_state_out, float *d_logits, int32_t *d_experts, float *d_stats, void *stream);

/* YGG_E_TOKEN if a step since the last call met a device token out of range, YGG_E_TIMEOUT if a step's bounded wait
 * for an asynchronous copy gave up (its results stay exact: the step then read the data from global memory), else
 * YGG_OK; the record is then cleared. Synchronises `stream`. */
YGG_API int ygg_fstatus(const ygg_fmodel *m, void *stream, int *status_out);

/* Free a float model; NULL is a no-op. */
YGG_API void ygg_ffree(ygg_fmodel *m);

/* Free the device memory of a model; NULL is a no-op. */
YGG_API void ygg_free(ygg_model *m);

/* Text of an error code. */
YGG_API const char *ygg_strerror(int code);

/* Library version string, and the sm architecture it was built for ("sm_100a"). */
YGG_API const char *ygg_version(void);

#ifdef __cplusplus
}
#endif

#endif
