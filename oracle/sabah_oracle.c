/*
 * CPU oracle for the routed-expert MUL_MAT_ID path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product links, loads or calls this
 * file; only the tests, the smoke check and bench.py's CPU-baseline leg do, as
 * the checker and as the timed CPU baseline.
 *
 * What it restates (reference file:line, paths inside Fovane/Sabah-MoE-Accelerator):
 *   - orc_dequant: the scalar ggml-order dequantizer sb_host_dequant
 *     (sabah/runtime/cuda/sabah_rt.cu:2233-2423) for the ten reference types,
 *     plus Q6_K, which the reference lacks; Q6_K follows gguf-py's
 *     quants.Q6_K.dequantize_blocks (integration/llama.cpp/gguf-py/gguf/quants.py:586).
 *     The float operations are done in the same order as gguf-py so results are
 *     bit-identical (build with -ffp-contract=off).
 *   - orc_mmid_f64: the float64 recomputation of one MUL_MAT_ID call that
 *     sb_selfcheck performs (sabah_rt.cu:3435-3492), over every (token, slot):
 *     dst[t][i][r] = sum_c W[ids[t][i]][r][c] * x[t][i % x_rows][c]
 *     with the v2 byte-stride contract (sabah_rt.cu:3494-3515).
 *   - orc_moe_block_f64: reference_block (sabah/runtime/executor.py:134-159):
 *     y = sum_k w_k * Wd[e_k] (silu(Wg[e_k] x) * Wu[e_k] x), silu(g) = g / (1 + exp(-g)).
 *   - orc_decode_f32: the timed CPU baseline; the same block math over a stack of
 *     layers in fp32 (row dequant + fp32 dot, as the reference's CPU path does),
 *     parallel over rows with pthreads; x_{L+1} = x_L + y_L between layers.
 *     A caller may pass the reference's own sabah_rt_host_dequant as the
 *     dequantizer, which makes this the reference's CPU path timed as-is.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "orc_tables.h"

#define ORC_Q5_1 7
#define ORC_Q8_0 8
#define ORC_Q4_K 12
#define ORC_Q5_K 13
#define ORC_Q6_K 14
#define ORC_IQ3_XXS 18
#define ORC_IQ4_NL 20
#define ORC_IQ3_S 21
#define ORC_IQ2_S 22
#define ORC_IQ4_XS 23
#define ORC_Q2_0 42

int orc_block_elems(int qt) {
    switch (qt) {
    case ORC_Q5_1: case ORC_Q8_0: case ORC_IQ4_NL: return 32;
    case ORC_Q2_0: return 64;
    case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: case ORC_IQ3_XXS:
    case ORC_IQ3_S: case ORC_IQ2_S: case ORC_IQ4_XS: return 256;
    }
    return 0;
}

int orc_block_bytes(int qt) {
    switch (qt) {
    case ORC_Q5_1: return 24;
    case ORC_Q8_0: return 34;
    case ORC_Q4_K: return 144;
    case ORC_Q5_K: return 176;
    case ORC_Q6_K: return 210;
    case ORC_IQ3_XXS: return 98;
    case ORC_IQ4_NL: return 18;
    case ORC_IQ3_S: return 110;
    case ORC_IQ2_S: return 82;
    case ORC_IQ4_XS: return 136;
    case ORC_Q2_0: return 18;
    }
    return 0;
}

/* IEEE binary16 -> binary32 by bit manipulation (sabah_rt.cu:2198-2221). */
static float orc_f16(const uint8_t *p) {
    uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ee = 113;               /* 127 - 15 + 1 */
            while (!(m & 0x400u)) { m <<= 1; --ee; }
            bits = sign | ((uint32_t)ee << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* 6-bit scale/min pair j of a K-quant 12-byte scale field (ggml get_scale_min_k4). */
static void orc_scale_min(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

static float orc_sgn(unsigned bits, int j) { return ((bits >> j) & 1u) ? -1.0f : 1.0f; }

/* Dequantize n elements (whole blocks) of type qt. Returns 0, or -1 for an
 * unknown type or a partial block. */
int orc_dequant(const uint8_t *x, float *y, int qt, int64_t n) {
    const int be = orc_block_elems(qt), bb = orc_block_bytes(qt);
    if (be == 0 || n < 0 || n % be) return -1;
    const int64_t nb = n / be;
    for (int64_t b = 0; b < nb; ++b, x += bb, y += be) {
        switch (qt) {
        case ORC_Q8_0: {
            const float d = orc_f16(x);
            for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)x[2 + j] * d;
            break;
        }
        case ORC_Q5_1: {
            const float d = orc_f16(x), m = orc_f16(x + 2);
            const uint32_t qh = (uint32_t)x[4] | ((uint32_t)x[5] << 8) | ((uint32_t)x[6] << 16) | ((uint32_t)x[7] << 24);
            const uint8_t *qs = x + 8;
            for (int j = 0; j < 16; ++j) {
                const int lo = (qs[j] & 15) | (((qh >> j) & 1) << 4);
                const int hi = (qs[j] >> 4) | (((qh >> (j + 16)) & 1) << 4);
                y[j] = d * (float)lo + m;
                y[j + 16] = d * (float)hi + m;
            }
            break;
        }
        case ORC_Q4_K: case ORC_Q5_K: {
            const float d = orc_f16(x), dmin = orc_f16(x + 2);
            const uint8_t *scl = x + 4;
            const uint8_t *qh = x + 16;                    /* Q5_K only */
            const uint8_t *ql = x + (qt == ORC_Q4_K ? 16 : 48);
            for (int s = 0; s < 8; ++s) {
                int sc, mn;
                orc_scale_min(s, scl, &sc, &mn);
                const float ds = d * (float)sc, dm = dmin * (float)mn;
                const uint8_t *q = ql + (s >> 1) * 32;
                for (int l = 0; l < 32; ++l) {
                    int v = (s & 1) ? (q[l] >> 4) : (q[l] & 15);
                    if (qt == ORC_Q5_K) v |= ((qh[l] >> s) & 1) << 4;
                    y[s * 32 + l] = ds * (float)v - dm;
                }
            }
            break;
        }
        case ORC_Q6_K: {
            /* ql[128] | qh[64] | scales[16] (int8) | d; 16 sub-blocks of 16 */
            const uint8_t *ql = x, *qh = x + 128;
            const int8_t *sc = (const int8_t *)(x + 192);
            const float d = orc_f16(x + 208);
            for (int h = 0; h < 2; ++h) {
                for (int l = 0; l < 32; ++l) {
                    const int q0 = ((ql[64 * h + l] & 15) | (((qh[32 * h + l] >> 0) & 3) << 4)) - 32;
                    const int q1 = ((ql[64 * h + l + 32] & 15) | (((qh[32 * h + l] >> 2) & 3) << 4)) - 32;
                    const int q2 = ((ql[64 * h + l] >> 4) | (((qh[32 * h + l] >> 4) & 3) << 4)) - 32;
                    const int q3 = ((ql[64 * h + l + 32] >> 4) | (((qh[32 * h + l] >> 6) & 3) << 4)) - 32;
                    const int e = 128 * h + l;
                    y[e + 0] = (d * (float)sc[(e + 0) / 16]) * (float)q0;
                    y[e + 32] = (d * (float)sc[(e + 32) / 16]) * (float)q1;
                    y[e + 64] = (d * (float)sc[(e + 64) / 16]) * (float)q2;
                    y[e + 96] = (d * (float)sc[(e + 96) / 16]) * (float)q3;
                }
            }
            break;
        }
        case ORC_IQ2_S: {
            /* d | qs[32] grid bytes | signs[32] | qh[8] | scales[8] */
            const float d = orc_f16(x);
            const uint8_t *qs = x + 2, *signs = x + 34, *qh = x + 66, *scl = x + 74;
            for (int ib = 0; ib < 8; ++ib) {
                const float db0 = d * (0.5f + (float)(scl[ib] & 15)) * 0.25f;
                const float db1 = d * (0.5f + (float)(scl[ib] >> 4)) * 0.25f;
                for (int l = 0; l < 4; ++l) {
                    const float db = l < 2 ? db0 : db1;
                    const unsigned gi = qs[4 * ib + l] | (((unsigned)qh[ib] >> (2 * l)) & 3u) << 8;
                    const uint64_t g = orc_iq2s_grid[gi];
                    for (int j = 0; j < 8; ++j)
                        y[32 * ib + 8 * l + j] = db * (float)((g >> (8 * j)) & 0xff) * orc_sgn(signs[4 * ib + l], j);
                }
            }
            break;
        }
        case ORC_IQ3_XXS: {
            /* d | qs[64] grid bytes | 8 x uint32 (4 x 7-bit sign index, 4-bit scale) */
            const float d = orc_f16(x);
            const uint8_t *qs = x + 2, *ss = x + 66;
            for (int ib = 0; ib < 8; ++ib) {
                const uint32_t a = (uint32_t)ss[4 * ib] | ((uint32_t)ss[4 * ib + 1] << 8) |
                                   ((uint32_t)ss[4 * ib + 2] << 16) | ((uint32_t)ss[4 * ib + 3] << 24);
                const float db = d * (0.5f + (float)(a >> 28)) * 0.5f;
                for (int l = 0; l < 4; ++l) {
                    const unsigned sg = orc_ksigns[(a >> (7 * l)) & 127];
                    const uint32_t g1 = orc_iq3xxs_grid[qs[8 * ib + 2 * l]];
                    const uint32_t g2 = orc_iq3xxs_grid[qs[8 * ib + 2 * l + 1]];
                    for (int j = 0; j < 4; ++j) {
                        y[32 * ib + 8 * l + j] = db * (float)((g1 >> (8 * j)) & 0xff) * orc_sgn(sg, j);
                        y[32 * ib + 8 * l + 4 + j] = db * (float)((g2 >> (8 * j)) & 0xff) * orc_sgn(sg, j + 4);
                    }
                }
            }
            break;
        }
        case ORC_IQ3_S: {
            /* d | qs[64] | qh[8] | signs[32] | scales[4] */
            const float d = orc_f16(x);
            const uint8_t *qs = x + 2, *qh = x + 66, *signs = x + 74, *scl = x + 106;
            for (int ib = 0; ib < 8; ++ib) {
                const float db = d * (float)(1 + 2 * ((scl[ib >> 1] >> (4 * (ib & 1))) & 15));
                for (int l = 0; l < 4; ++l) {
                    const unsigned i1 = qs[8 * ib + 2 * l] | (((unsigned)qh[ib] >> (2 * l)) & 1u) << 8;
                    const unsigned i2 = qs[8 * ib + 2 * l + 1] | (((unsigned)qh[ib] >> (2 * l + 1)) & 1u) << 8;
                    const uint32_t g1 = orc_iq3s_grid[i1], g2 = orc_iq3s_grid[i2];
                    const unsigned sg = signs[4 * ib + l];
                    for (int j = 0; j < 4; ++j) {
                        y[32 * ib + 8 * l + j] = db * (float)((g1 >> (8 * j)) & 0xff) * orc_sgn(sg, j);
                        y[32 * ib + 8 * l + 4 + j] = db * (float)((g2 >> (8 * j)) & 0xff) * orc_sgn(sg, j + 4);
                    }
                }
            }
            break;
        }
        case ORC_IQ4_NL: {
            const float d = orc_f16(x);
            for (int j = 0; j < 16; ++j) {
                y[j] = d * (float)orc_kvalues_iq4nl[x[2 + j] & 15];
                y[j + 16] = d * (float)orc_kvalues_iq4nl[x[2 + j] >> 4];
            }
            break;
        }
        case ORC_IQ4_XS: {
            /* d | scales_h (u16) | scales_l[4] | qs[128] */
            const float d = orc_f16(x);
            const unsigned sh = (unsigned)x[2] | ((unsigned)x[3] << 8);
            const uint8_t *sl = x + 4, *qs = x + 8;
            for (int ib = 0; ib < 8; ++ib) {
                const int ls = (int)(((sl[ib >> 1] >> (4 * (ib & 1))) & 15) | (((sh >> (2 * ib)) & 3) << 4));
                const float dl = d * (float)(ls - 32);
                for (int j = 0; j < 16; ++j) {
                    y[32 * ib + j] = dl * (float)orc_kvalues_iq4nl[qs[16 * ib + j] & 15];
                    y[32 * ib + 16 + j] = dl * (float)orc_kvalues_iq4nl[qs[16 * ib + j] >> 4];
                }
            }
            break;
        }
        case ORC_Q2_0: {
            const float d = orc_f16(x);
            for (int j = 0; j < 64; ++j) {
                const int q = (x[2 + (j >> 2)] >> (2 * (j & 3))) & 3;
                y[j] = ((float)q - 1.0f) * d;
            }
            break;
        }
        default:
            return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* fp64 MUL_MAT_ID, v2 stride contract (all strides in bytes).               */
/* dst is dense: dst[(t * n_ids + i) * rows + r].                            */
/* Returns 0, -1 for an id outside [0, n_experts), -2 for a bad geometry.    */
/* ------------------------------------------------------------------------ */
int orc_mmid_f64(const uint8_t *source, size_t expert_stride, size_t row_stride,
                 const float *x, size_t x_id_stride, int x_rows, size_t x_token_stride,
                 const int32_t *ids, size_t ids_id_stride, size_t ids_token_stride,
                 int n_ids, int n_tokens, double *dst, int rows, int k, int n_experts, int qt) {
    if (k <= 0 || rows <= 0 || n_ids <= 0 || n_tokens < 0 || (x_rows != 1 && x_rows != n_ids)) return -2;
    if (orc_block_elems(qt) == 0 || k % orc_block_elems(qt)) return -2;
    float *w = (float *)malloc((size_t)k * sizeof(float));
    if (!w) return -2;
    for (int t = 0; t < n_tokens; ++t) {
        for (int i = 0; i < n_ids; ++i) {
            const int e = *(const int32_t *)((const uint8_t *)ids + (size_t)t * ids_token_stride + (size_t)i * ids_id_stride);
            if (e < 0 || e >= n_experts) { free(w); return -1; }
            const float *xr = (const float *)((const uint8_t *)x + (size_t)(i % x_rows) * x_id_stride + (size_t)t * x_token_stride);
            for (int r = 0; r < rows; ++r) {
                orc_dequant(source + (size_t)e * expert_stride + (size_t)r * row_stride, w, qt, k);
                double acc = 0.0;
                for (int c = 0; c < k; ++c) acc += (double)w[c] * (double)xr[c];
                dst[((size_t)t * n_ids + i) * rows + r] = acc;
            }
        }
    }
    free(w);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* fp64 fused MoE block (executor.py reference_block), one token.            */
/* gate/up/down: per-slot expert base pointers; rows are contiguous.         */
/* ------------------------------------------------------------------------ */
int orc_moe_block_f64(const uint8_t *const *gate, const uint8_t *const *up, const uint8_t *const *down,
                      const float *w, const float *x, double *out, int d_model, int ff, int n_used,
                      int qt_gate, int qt_up, int qt_down, double *h_out) {
    const size_t rbg = (size_t)(d_model / orc_block_elems(qt_gate)) * orc_block_bytes(qt_gate);
    const size_t rbu = (size_t)(d_model / orc_block_elems(qt_up)) * orc_block_bytes(qt_up);
    const size_t rbd = (size_t)(ff / orc_block_elems(qt_down)) * orc_block_bytes(qt_down);
    float *row = (float *)malloc((size_t)(d_model > ff ? d_model : ff) * sizeof(float));
    double *h = (double *)malloc((size_t)ff * sizeof(double));
    if (!row || !h) { free(row); free(h); return -2; }
    for (int i = 0; i < d_model; ++i) out[i] = 0.0;
    for (int e = 0; e < n_used; ++e) {
        for (int j = 0; j < ff; ++j) {
            double g = 0.0, u = 0.0;
            orc_dequant(gate[e] + (size_t)j * rbg, row, qt_gate, d_model);
            for (int c = 0; c < d_model; ++c) g += (double)row[c] * (double)x[c];
            orc_dequant(up[e] + (size_t)j * rbu, row, qt_up, d_model);
            for (int c = 0; c < d_model; ++c) u += (double)row[c] * (double)x[c];
            h[j] = (g / (1.0 + exp(-g))) * u;
            if (h_out) h_out[(size_t)e * ff + j] = h[j];
        }
        for (int i = 0; i < d_model; ++i) {
            orc_dequant(down[e] + (size_t)i * rbd, row, qt_down, ff);
            double acc = 0.0;
            for (int c = 0; c < ff; ++c) acc += (double)row[c] * h[c];
            out[i] += (double)w[e] * acc;
        }
    }
    free(row);
    free(h);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Timed CPU baseline: fp32 multi-layer decode, pthreads over rows.          */
/* ------------------------------------------------------------------------ */
typedef int (*orc_dequant_fn)(const void *src, float *dst, int qt, int n);

static int orc_dequant_int(const void *src, float *dst, int qt, int n) {
    return orc_dequant((const uint8_t *)src, dst, qt, n);
}

typedef struct {
    /* problem */
    const uint8_t *const *gate_base, *const *up_base, *const *down_base;
    size_t gu_expert_stride, d_expert_stride, rbgu, rbd;
    int qt_gu, qt_d, d_model, ff, n_used, n_layers;
    const int32_t *ids;
    const float *wts;
    float *x, *h, *y;
    orc_dequant_fn dq;
    /* threading */
    int n_threads;
    pthread_barrier_t bar;
    int error;
} orc_decode_job;

typedef struct { orc_decode_job *job; int tid; } orc_worker_arg;

static void *orc_decode_worker(void *p) {
    orc_worker_arg *a = (orc_worker_arg *)p;
    orc_decode_job *J = a->job;
    const int tid = a->tid, nt = J->n_threads;
    const int dm = J->d_model, ff = J->ff, nu = J->n_used;
    float *row = (float *)malloc((size_t)(dm > ff ? dm : ff) * sizeof(float));
    for (int L = 0; L < J->n_layers; ++L) {
        const int32_t *ids = J->ids + (size_t)L * nu;
        const float *w = J->wts + (size_t)L * nu;
        /* phase 1: h[e][j] = silu(<Wg,x>) * <Wu,x>, split over (e, j) */
        for (int idx = tid; idx < nu * ff; idx += nt) {
            const int e = idx / ff, j = idx % ff;
            const uint8_t *g = J->gate_base[L] + (size_t)ids[e] * J->gu_expert_stride + (size_t)j * J->rbgu;
            const uint8_t *u = J->up_base[L] + (size_t)ids[e] * J->gu_expert_stride + (size_t)j * J->rbgu;
            float sg = 0.f, su = 0.f;
            if (J->dq(g, row, J->qt_gu, dm)) J->error = 1;
            for (int c = 0; c < dm; ++c) sg += row[c] * J->x[c];
            if (J->dq(u, row, J->qt_gu, dm)) J->error = 1;
            for (int c = 0; c < dm; ++c) su += row[c] * J->x[c];
            J->h[(size_t)e * ff + j] = (sg / (1.0f + expf(-sg))) * su;
        }
        pthread_barrier_wait(&J->bar);
        /* phase 2: y[i] = sum_e w[e] <Wd[e][i], h[e]>, fixed expert order */
        for (int i = tid; i < dm; i += nt) {
            float tot = 0.f;
            for (int e = 0; e < nu; ++e) {
                const uint8_t *d = J->down_base[L] + (size_t)ids[e] * J->d_expert_stride + (size_t)i * J->rbd;
                if (J->dq(d, row, J->qt_d, ff)) J->error = 1;
                float a = 0.f;
                for (int c = 0; c < ff; ++c) a += row[c] * J->h[(size_t)e * ff + c];
                tot += w[e] * a;
            }
            J->y[i] = tot;
        }
        pthread_barrier_wait(&J->bar);
        /* residual: x <- x + y */
        for (int i = tid; i < dm; i += nt) J->x[i] += J->y[i];
        pthread_barrier_wait(&J->bar);
    }
    free(row);
    return NULL;
}

/* x is updated in place (x_{L+1} = x_L + y_L). ids/wts are [n_layers][n_used].
 * dq may be NULL (use orc_dequant) or the reference's sabah_rt_host_dequant. */
int orc_decode_f32(const uint8_t *const *gate_base, const uint8_t *const *up_base,
                   const uint8_t *const *down_base, size_t gu_expert_stride, size_t d_expert_stride,
                   int qt_gu, int qt_d, int n_layers, const int32_t *ids, const float *wts, float *x,
                   int d_model, int ff, int n_used, int n_threads, void *dq) {
    if (n_threads < 1) n_threads = 1;
    orc_decode_job J;
    memset(&J, 0, sizeof(J));
    J.gate_base = gate_base; J.up_base = up_base; J.down_base = down_base;
    J.gu_expert_stride = gu_expert_stride; J.d_expert_stride = d_expert_stride;
    J.rbgu = (size_t)(d_model / orc_block_elems(qt_gu)) * orc_block_bytes(qt_gu);
    J.rbd = (size_t)(ff / orc_block_elems(qt_d)) * orc_block_bytes(qt_d);
    J.qt_gu = qt_gu; J.qt_d = qt_d; J.d_model = d_model; J.ff = ff; J.n_used = n_used;
    J.n_layers = n_layers; J.ids = ids; J.wts = wts; J.x = x;
    J.dq = dq ? (orc_dequant_fn)dq : orc_dequant_int;
    J.n_threads = n_threads;
    J.h = (float *)malloc((size_t)n_used * ff * sizeof(float));
    J.y = (float *)malloc((size_t)d_model * sizeof(float));
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)n_threads);
    orc_worker_arg *args = (orc_worker_arg *)malloc(sizeof(orc_worker_arg) * (size_t)n_threads);
    pthread_barrier_init(&J.bar, NULL, (unsigned)n_threads);
    for (int t = 0; t < n_threads; ++t) {
        args[t].job = &J; args[t].tid = t;
        pthread_create(&th[t], NULL, orc_decode_worker, &args[t]);
    }
    for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
    pthread_barrier_destroy(&J.bar);
    free(th); free(args); free(J.h); free(J.y);
    return J.error ? -1 : 0;
}
