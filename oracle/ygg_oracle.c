/* TEST INFRASTRUCTURE ONLY -- the CPU checker for the CUDA path, never the product and never linked into it.
 *
 * A plain-C, scalar restatement of the reference int8 step (cpu/ygg.cpp, bit-exact with cpu/export.py:268-316
 * int_forward) over the reference's own YGG1 file bytes. It exposes what the reference kernel keeps internal (the
 * leaf each layer routes to, the int8 states) so that the GPU path can be compared on routes and states as well as
 * logits. Pinned against the reference: tests/test_oracle.py checks it against golden digests of the reference's
 * int_forward / ygg outputs (tests/golden/make_golden.py) on every shape of the reference's kernel test.
 *
 * Arithmetic rules copied in meaning (not code) from cpu/ygg.cpp, compiled with -ffp-contract=off:
 *   integer dots are exact (u8 storage w + 128 with the 128 * sum correction gives the signed dot);
 *   f32 ops are single-rounded in the reference's order; rint is round-half-even (cvtps_epi32 / np.rint).
 */
#define _POSIX_C_SOURCE 200112L
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define MAX_LAYERS 8
#define CLASS_PAD 32

typedef struct {
    const uint8_t *rec; int rec_bytes;
    int off_a, off_u, off_p, off_t, off_f, off_c, off_s;   /* record parts, -1 absent */
    int table_stride;                                      /* bytes per token row of T_r; 0 for the token layer */
    const uint8_t *q;                                      /* unembedding u8 [R/4][VP][4] */
    float readout_scale, unembed_scale, rms_eps, layer_input_scale;
    const uint8_t *w; const float *thr;                    /* router u8 [E][n], thresholds f32 [V][E] */
    const uint8_t *vl; const float *mv;                    /* layer-input down projection u8 [RG][n/4][16][4] */
    const float *mulv, *r2b, *mzl, *sqv;                   /* group scales (NULL: per tensor) */
    const int8_t *vt; const float *mt;                     /* factored input: token codes, token scale */
} OLayer;

typedef struct {
    int L, n, b, V, D, R, R2, k, shift, E, VP;
    const float *head_b;
    OLayer y[MAX_LAYERS];
    uint8_t *blob;                                          /* copy of the array section, 64-aligned */
} orc_model;

typedef struct { char name[32]; int64_t off, bytes; } Entry;

static const uint8_t *find(const Entry *tab, int na, const uint8_t *base, const char *name) {
    for (int i = 0; i < na; i++) if (!strncmp(tab[i].name, name, 32)) return base + tab[i].off;
    return NULL;
}

/* YGG1 parse: header and limits as cpu/ygg.cpp:137-148, array binding as cpu/ygg.cpp:173-220. Beyond the reference's
 * limits it admits this repository's one format extension, d_state 96 with readout rank 12 (stored in the rank-16
 * readout layout with zero rows 12-15), which int_forward (cpu/export.py:268-316) computes at any shape. */
orc_model *orc_load(const uint8_t *bytes, size_t nbytes, char *err, int errlen) {
    int32_t h[12];
    if (nbytes < 52 || memcmp(bytes, "YGG1", 4)) { snprintf(err, errlen, "not a model file"); return NULL; }
    memcpy(h, bytes + 4, 48);
    const int L = h[0], n = h[1], b = h[2], V = h[3], D = h[4], R = h[5], R2 = h[6], na = h[11];
    const int ok = (n == 64 || n == 96 || n == 128 || n == 256) && (b == 8 || b == 16) &&
                   (R == 8 || R == 12 || R == 16 || R == 32) &&
                   R2 <= 64 && R2 % 4 == 0 && L >= 1 && L <= MAX_LAYERS && V <= 256 && D <= 16 &&
                   (L == 1 || D >= 1) && h[7] == 0;
    if (!ok) { snprintf(err, errlen, "unsupported model"); return NULL; }
    if (nbytes < 52 + (size_t)na * 48) { snprintf(err, errlen, "short array table"); return NULL; }
    Entry *tab = (Entry *)malloc(sizeof(Entry) * (na ? na : 1));
    memcpy(tab, bytes + 52, sizeof(Entry) * na);
    size_t pos = 52 + (size_t)na * 48; pos += (64 - pos % 64) % 64;
    const size_t sz = nbytes - pos;
    orc_model *m = (orc_model *)calloc(1, sizeof(orc_model));
    if (posix_memalign((void **)&m->blob, 64, sz + 128)) { free(tab); free(m); snprintf(err, errlen, "oom"); return NULL; }
    memcpy(m->blob, bytes + pos, sz); memset(m->blob + sz, 0, 128);
    for (int i = 0; i < na; i++)
        if (tab[i].off < 0 || tab[i].bytes < 0 || (size_t)(tab[i].off + tab[i].bytes) > sz) {
            snprintf(err, errlen, "array %.32s out of the file", tab[i].name); free(tab); free(m->blob); free(m); return NULL;
        }
    m->L = L; m->n = n; m->b = b; m->V = V; m->D = D; m->R = R; m->R2 = R2; m->k = h[9]; m->shift = h[10];
    m->E = 1 << D; m->VP = (V + CLASS_PAD - 1) / CLASS_PAD * CLASS_PAD;
    m->head_b = (const float *)find(tab, na, m->blob, "head_b");
    if (!m->head_b) { snprintf(err, errlen, "missing head_b"); goto fail; }
    for (int l = 0; l < L; l++) {
        OLayer *y = &m->y[l];
        char nm[40];
#define GET(tag) (snprintf(nm, sizeof nm, "l%d_%s", l, tag), find(tab, na, m->blob, nm))
        const int32_t *meta = (const int32_t *)GET("meta");
        y->rec = GET("rec"); y->q = GET("Q");
        const float *sc = (const float *)GET("scal");
        if (!meta || !y->rec || !y->q || !sc) { snprintf(err, errlen, "layer %d: missing arrays", l); goto fail; }
        y->rec_bytes = meta[0]; y->off_a = meta[1]; y->off_u = meta[2]; y->off_p = meta[3]; y->off_t = meta[4];
        y->vt = (const int8_t *)GET("vt");
        y->off_f = y->off_c = y->off_s = -1;
        if (y->vt) { y->off_f = meta[5]; y->off_c = meta[6]; y->off_s = meta[7]; y->mt = (const float *)GET("mT"); }
        y->table_stride = l == 0 ? 0 : 2 * n;
        y->readout_scale = sc[0]; y->unembed_scale = sc[1]; y->rms_eps = sc[2]; y->layer_input_scale = sc[3];
        y->mzl = (const float *)GET("mzl"); y->sqv = (const float *)GET("sqv");
        if (l > 0) {
            y->w = GET("w"); y->thr = (const float *)GET("thr");
            if (!y->w || !y->thr) { snprintf(err, errlen, "layer %d: missing router", l); goto fail; }
            if (R2) { y->vl = GET("vl"); y->mv = (const float *)GET("mv"); }
            y->mulv = (const float *)GET("mulv"); y->r2b = (const float *)GET("r2b");
        }
#undef GET
    }
    free(tab);
    return m;
fail:
    free(tab); free(m->blob); free(m); return NULL;
}

void orc_free(orc_model *m) { if (m) { free(m->blob); free(m); } }

void orc_info(const orc_model *m, int32_t *out) {
    out[0] = m->L; out[1] = m->n; out[2] = m->b; out[3] = m->V; out[4] = m->D; out[5] = m->R; out[6] = m->R2;
    out[7] = m->k; out[8] = m->shift; out[9] = m->E; out[10] = m->VP; out[11] = m->y[1 < m->L ? 1 : 0].vt != NULL;
}

static inline int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : v > hi ? hi : v; }
/* f32 -> int32 round half to even, as _mm512_cvtps_epi32 under the default rounding mode: NaN and values outside
 * the int32 range give 0x80000000 (the x86 "integer indefinite"), which the callers then clamp */
static inline int32_t rne(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)rintf(v);
}

/* rho = 1 / sqrt(f32(sum q^2) * (1/n) + eps) (cpu/ygg.cpp:248-255); group scales: sequential f32 sum over groups of
 * 16 of r2[g] * f32(S_g) (cpu/ygg.cpp:257-266). */
static float rms_rho(const orc_model *m, const OLayer *y, const int8_t *qb) {
    const int n = m->n;
    if (y->r2b) {
        float s = 0.0f;
        for (int g = 0; g < n / 16; g++) {
            int32_t sg = 0;
            for (int j = 0; j < 16; j++) sg += (int32_t)qb[16 * g + j] * qb[16 * g + j];
            const float t = y->r2b[g] * (float)sg;
            s = s + t;
        }
        const float a = s * (1.0f / (float)n);
        return 1.0f / sqrtf(a + y->rms_eps);
    }
    int32_t ss = 0;
    for (int j = 0; j < n; j++) ss += (int32_t)qb[j] * qb[j];
    const float a = (float)ss * (1.0f / (float)n);
    return 1.0f / sqrtf(a + y->rms_eps);
}

/* heap-order descent, right iff f32(w_ix . qb) * rho > thr[x][ix] (cpu/ygg.cpp:271-280) */
static int route(const orc_model *m, const OLayer *y, int x, const int8_t *qb, float rho) {
    const int n = m->n;
    int ix = 1;
    for (int d = 0; d < m->D; d++) {
        const uint8_t *w = y->w + (size_t)ix * n;
        int32_t dot = 0;
        for (int j = 0; j < n; j++) dot += ((int32_t)w[j] - 128) * qb[j];
        const float s = (float)dot * rho;
        ix = 2 * ix + (s > y->thr[(size_t)x * m->E + ix]);
    }
    return ix - m->E;
}

/* zl[k] = clamp(rint((f32(V'_k . qb) * mv[k]) * rho), +-127) (cpu/ygg.cpp:285-296) */
static void layer_input(const orc_model *m, const OLayer *y, const int8_t *qb, float rho, int8_t *zl) {
    const int n = m->n;
    for (int k = 0; k < m->R2; k++) {
        const int gi = k / 16, kk = k % 16;
        int32_t a = 0;
        for (int j = 0; j < n; j++)
            a += ((int32_t)y->vl[((size_t)(gi * (n / 4) + j / 4) * 16 + kk) * 4 + j % 4] - 128) * qb[j];
        float zf = (float)a * y->mv[k];
        zf = zf * rho;
        zl[k] = (int8_t)clampi(rne(zf), -127, 127);
    }
}

/* q <- sat8((A16 q + 2^(shift-1)) >> shift + input + rint(f32(U' zl) m_ul)) (cpu/ygg.cpp:312-389); acc_out (n) or
 * NULL receives the int32 accumulator before the saturation (the `acc` that cpu/ygg.cpp:388 narrows with
 * cvtsepi32_epi8; `drive` in cpu/export.py:307-310) */
static void update(const orc_model *m, const OLayer *y, int r, int x, int8_t *q, const int8_t *zl, int32_t *acc_out) {
    const int n = m->n, b = m->b;
    const uint8_t *rec = y->rec + (size_t)r * y->rec_bytes;
    const int16_t *A = (const int16_t *)(rec + y->off_a);
    int32_t acc[256];
    for (int i = 0; i < n; i++) {
        const int gg = i / 16, ii = i % 16, c0 = (i / b) * b;
        int32_t s = 0;
        for (int jj = 0; jj < b; jj++)
            s += (int32_t)A[((gg * (b / 2) + jj / 2) * 16 + ii) * 2 + jj % 2] * q[c0 + jj];
        acc[i] = (s + (1 << (m->shift - 1))) >> m->shift;   /* arithmetic shift */
    }
    if (y->vt) {   /* factored: rint(f32(U_r v[x]) * f32(su_r * mT[i])) + c_r[i] (cpu/ygg.cpp:339-358) */
        const uint8_t *U = rec + y->off_f;
        const int8_t *v = y->vt + (size_t)x * m->k;
        const int16_t *C = (const int16_t *)(rec + y->off_c);
        float su; memcpy(&su, rec + y->off_s, 4);
        for (int i = 0; i < n; i++) {
            int32_t lt = 0;
            for (int kk = 0; kk < m->k; kk++) lt += ((int32_t)U[((size_t)(kk / 4) * n + i) * 4 + kk % 4] - 128) * v[kk];
            const float mul = su * y->mt[i];
            acc[i] += rne((float)lt * mul) + C[i];
        }
    } else {       /* table row T_r[x] (cpu/ygg.cpp:334-337) */
        const int16_t *T = (const int16_t *)(rec + y->off_t + (size_t)x * y->table_stride);
        for (int i = 0; i < n; i++) acc[i] += T[i];
    }
    if (zl) {      /* (cpu/ygg.cpp:360-377) */
        const uint8_t *U = rec + y->off_u;
        for (int i = 0; i < n; i++) {
            int32_t la = 0;
            for (int kk = 0; kk < m->R2; kk++) la += ((int32_t)U[((size_t)(kk / 4) * n + i) * 4 + kk % 4] - 128) * zl[kk];
            const float mu = y->mulv ? y->mulv[i] : y->layer_input_scale;
            acc[i] += rne((float)la * mu);
        }
    }
    if (acc_out) memcpy(acc_out, acc, 4 * (size_t)n);
    for (int i = 0; i < n; i++) q[i] = (int8_t)clampi(acc[i], -128, 127);
}

/* zq = clamp(rint(f32(P_r q) * m_z), +-127); lg = base + f32(Q zq) * s (cpu/ygg.cpp:395-435) */
static void readout(const orc_model *m, const OLayer *y, int r, const int8_t *q, float *lg, const float *base) {
    const int n = m->n, R = m->R, VP = m->VP;
    const uint8_t *P = y->rec + (size_t)r * y->rec_bytes + y->off_p;
    int8_t zq[32];
    for (int rr = 0; rr < R; rr++) {
        int32_t z = 0;
        for (int i = 0; i < n; i++) {
            size_t idx;
            if (R == 8) idx = ((size_t)(i / 8) * 16 + 2 * rr + (i % 8) / 4) * 4 + i % 4;
            else idx = ((size_t)((rr / 16) * (n / 4) + i / 4) * 16 + rr % 16) * 4 + i % 4;
            z += ((int32_t)P[idx] - 128) * q[i];
        }
        const float mz = y->mzl ? y->mzl[(size_t)r * (R == 8 ? 16 : R) + (R == 8 ? 2 * rr : rr)] : y->readout_scale;
        zq[rr] = (int8_t)clampi(rne((float)z * mz), -127, 127);
    }
    for (int c = 0; c < VP; c++) {
        int32_t a = 0;
        for (int kk = 0; kk < R; kk++) a += ((int32_t)y->q[((size_t)(kk / 4) * VP + c) * 4 + kk % 4] - 128) * zq[kk];
        const float s = y->sqv ? y->sqv[c] : y->unembed_scale;
        const float t = (float)a * s;
        lg[c] = base[c] + t;
    }
}

/* one token of one stream over every layer (cpu/ygg.cpp:441-459); q: L*n int8, lg: VP floats; routes (L) and acc
 * (L*n, the accumulators before saturation) or NULL */
static void step1(const orc_model *m, int x, int8_t *q, float *lg, int32_t *routes, int32_t *acc) {
    for (int l = 0; l < m->L; l++) {
        const OLayer *y = &m->y[l];
        int8_t *ql = q + (size_t)l * m->n;
        int32_t *al = acc ? acc + (size_t)l * m->n : NULL;
        int r = x;
        if (l > 0) {
            const int8_t *qb = ql - m->n;
            const float rho = rms_rho(m, y, qb);
            r = route(m, y, x, qb, rho);
            if (m->R2) {
                int8_t zl[64];
                layer_input(m, y, qb, rho, zl);
                update(m, y, r, x, ql, zl, al);
            } else update(m, y, r, x, ql, NULL, al);
        } else update(m, y, r, x, ql, NULL, al);
        if (routes) routes[l] = r;
        readout(m, y, r, ql, lg, l == 0 ? m->head_b : lg);
    }
}

static int check_tokens(const orc_model *m, size_t cnt, const int32_t *tok) {
    for (size_t i = 0; i < cnt; i++) if (tok[i] < 0 || tok[i] >= m->V) return -1;
    return 0;
}

/* one step of B streams: state (B, L, n) in/out, logits (B, V) or NULL, routes (B, L) or NULL, acc (B, L, n) or NULL
 * (the int32 accumulators before saturation) */
int orc_step(const orc_model *m, int B, const int32_t *tok, int8_t *state, float *logits, int32_t *routes,
             int32_t *acc) {
    if (check_tokens(m, (size_t)B, tok)) return -1;
    float lg[256];
    for (int s = 0; s < B; s++) {
        step1(m, tok[s], state + (size_t)s * m->L * m->n, lg, routes ? routes + (size_t)s * m->L : NULL,
              acc ? acc + (size_t)s * m->L * m->n : NULL);
        if (logits) memcpy(logits + (size_t)s * m->V, lg, 4 * (size_t)m->V);
    }
    return 0;
}

/* windows of tokens (S, T) from a zero state each: logits (S, T, V), routes (S, T, L) or NULL, acc (S, T, L, n) or
 * NULL (cpu/ygg.cpp:500-512, the logits command) */
int orc_logits(const orc_model *m, int S, int T, const int32_t *tok, float *logits, int32_t *routes, int32_t *acc) {
    if (check_tokens(m, (size_t)S * T, tok)) return -1;
    int8_t *q = (int8_t *)calloc((size_t)m->L * m->n, 1);
    float lg[256];
    for (int s = 0; s < S; s++) {
        memset(q, 0, (size_t)m->L * m->n);
        for (int t = 0; t < T; t++) {
            const size_t i = (size_t)s * T + t;
            step1(m, tok[i], q, lg, routes ? routes + i * m->L : NULL, acc ? acc + i * m->L * m->n : NULL);
            memcpy(logits + i * m->V, lg, 4 * (size_t)m->V);
        }
    }
    free(q);
    return 0;
}

/* bits of tokens[:, 1:] given the tokens before them, per row, in f64 (the NLL of cpu/ygg.cpp:513-517 over the
 * rows of yggdrasil/inference.py:179-188); state (S, L, n) in/out, NULL: zero */
int orc_score(const orc_model *m, int S, int T, const int32_t *tok, int8_t *state, double *bits) {
    if (check_tokens(m, (size_t)S * T, tok)) return -1;
    int8_t *own = (int8_t *)calloc((size_t)m->L * m->n, 1);
    float lg[256];
    for (int s = 0; s < S; s++) {
        int8_t *q = state ? state + (size_t)s * m->L * m->n : own;
        if (!state) memset(own, 0, (size_t)m->L * m->n);
        double nll = 0.0;
        for (int t = 0; t + 1 < T; t++) {
            step1(m, tok[(size_t)s * T + t], q, lg, NULL, NULL);
            double mx = -1e300;
            for (int c = 0; c < m->V; c++) mx = lg[c] > mx ? lg[c] : mx;
            double se = 0.0;
            for (int c = 0; c < m->V; c++) se += exp((double)lg[c] - mx);
            nll += log(se) + mx - (double)lg[tok[(size_t)s * T + t + 1]];
        }
        bits[s] = nll / log(2.0);
    }
    free(own);
    return 0;
}
