/*
 * ref_harness.c -- TEST INFRASTRUCTURE ONLY (linked into oracle/_ref/libggml_ref_*.so by
 * oracle/ref.mk, together with the reference's vendored ggml + ggml-cpu sources).
 *
 * Builds the reference's *unfused* MLA decode-attention graph -- the flag-OFF op sequence of
 * engine/m1_layer.cpp:437-502 (wk_b mul_mat over the permuted nope view, concat with the roped
 * q_pe, K.Q mul_mat, soft_max_ext with the mask and kq_scale, cont(transpose(V)), V^T.P mul_mat,
 * wv_b mul_mat) -- with the reference's own ggml API, at a run-time geometry, and computes it on
 * the reference's own ggml-cpu backend.  This is the numerics oracle by the reference's own design
 * (its fused ops abort on the CPU, ggml-cpu.c:2064-2082) and the timed CPU baseline.
 *
 * Geometry (ggml ne[] order):
 *   q      F32 [dq, H]         dq = nope + rope, head stride dq floats (the g_q layout)
 *   wk_b   F16 [nope, R, H]    R = latent (kv_lora_rank)
 *   kcache F16 [R + rope, N]
 *   mask   F32 [N, 1]
 *   wv_b   F16 [R, V, H]
 * Taps: q_abs F32 [R, H] (after the permute back), attn (g_kqv) F32 [R, 1, H], out F32 [V, 1, H].
 * wk_b / wv_b are F16 (BASELINE) or Q8_0 (the Mistral-Small-4 geometry, engine/m1_layer.h:47-55),
 * passed as raw ggml bytes.
 *
 * A second graph, ref_kvw_*, is the flag-OFF KV-write sequence of engine/m1_layer.cpp:422-460
 * (the ops GGML_OP_M4_PHASE selector 0 replaces): wkv_a_mqa mul_mat (Q8_0) -> split into
 * {kv_cmpr | k_pe} -> rope_ext(k_pe, pos) -> rms_norm(kv_cmpr) * kv_a_norm -> concat ->
 * set_rows(kcache, Kcur, kidx).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ggml.h"
#include "ggml-cpu.h"

typedef struct ref_mla {
    int H, nope, rope, R, V;
    int64_t N;
    int n_threads;
    struct ggml_context * ctx;
    struct ggml_cgraph * gf;
    struct ggml_threadpool * tp;
    uint8_t * work;
    size_t work_size;
    struct ggml_tensor *q, *wkb, *kc, *mask, *wvb;
    struct ggml_tensor *q_abs, *qcur, *kqv, *out;
} ref_mla;

/* Build the graph once; inputs are then written with ref_mla_set_* and computed repeatedly.
 * wtype: the ggml type of wk_b and wv_b (GGML_TYPE_F16 or GGML_TYPE_Q8_0). */
ref_mla * ref_mla_create_typed(int H, int nope, int rope, int R, int V, int64_t N,
                               float kq_scale, int n_threads, int wtype) {
    if (wtype != GGML_TYPE_F16 && wtype != GGML_TYPE_Q8_0) return NULL;
    if (H <= 0 || nope <= 0 || rope < 0 || R <= 0 || V <= 0 || N <= 0 || n_threads <= 0)
        return NULL;
    ref_mla * m = (ref_mla *) calloc(1, sizeof(ref_mla));
    m->H = H; m->nope = nope; m->rope = rope; m->R = R; m->V = V; m->N = N;
    m->n_threads = n_threads;
    const int D = R + rope, dq = nope + rope;

    size_t bytes = 0;
    bytes += (size_t) dq * H * 4;                 /* q */
    bytes += (size_t) nope * R * H * 2;           /* wk_b */
    bytes += (size_t) D * N * 2;                  /* kcache */
    bytes += (size_t) N * 4;                      /* mask */
    bytes += (size_t) R * V * H * 2;              /* wv_b */
    bytes += (size_t) R * H * 4 * 2;              /* q_abs (+permute is a view) */
    bytes += (size_t) D * H * 4;                  /* qcur */
    bytes += (size_t) N * H * 4 * 2;              /* kq, softmax */
    bytes += (size_t) N * R * 2;                  /* vT (cont) */
    bytes += (size_t) R * H * 4 + (size_t) V * H * 4;
    bytes += 64 * ggml_tensor_overhead() + ggml_graph_overhead() + (1u << 20);

    struct ggml_init_params ip = { bytes, NULL, false };
    m->ctx = ggml_init(ip);
    if (!m->ctx) { free(m); return NULL; }
    struct ggml_context * ctx = m->ctx;

    m->q    = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, dq, H);
    m->wkb  = ggml_new_tensor_3d(ctx, (enum ggml_type) wtype, nope, R, H);
    m->kc   = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, D, N);
    m->mask = ggml_new_tensor_4d(ctx, GGML_TYPE_F32, N, 1, 1, 1);
    m->wvb  = ggml_new_tensor_3d(ctx, (enum ggml_type) wtype, R, V, H);

    /* m1_layer.cpp:390-392 (q3 / q_nope / q_pe views), with q_pe already roped by the caller */
    struct ggml_tensor * q3 = ggml_reshape_3d(ctx, m->q, dq, H, 1);
    struct ggml_tensor * q_nope = ggml_view_3d(ctx, q3, nope, H, 1, q3->nb[1], q3->nb[2], 0);
    struct ggml_tensor * q_pe = ggml_view_3d(ctx, q3, rope, H, 1, q3->nb[1], q3->nb[2],
                                             ggml_row_size(q3->type, nope));
    /* m1_layer.cpp:444-446: the absorption */
    struct ggml_tensor * q_nope_perm = ggml_permute(ctx, q_nope, 0, 2, 1, 3);
    struct ggml_tensor * qabs = ggml_mul_mat(ctx, m->wkb, q_nope_perm);      /* [R, 1, H] */
    m->q_abs = ggml_cont(ctx, ggml_permute(ctx, qabs, 0, 2, 1, 3));          /* [R, H, 1] tap */
    /* m1_layer.cpp:452: Qcur = concat(absorbed nope, roped pe) */
    m->qcur = ggml_concat(ctx, ggml_permute(ctx, qabs, 0, 2, 1, 3), q_pe, 0); /* [D, H, 1] */

    /* m1_layer.cpp:477-494: the non-flash-attn attention */
    struct ggml_tensor * q4 = ggml_view_4d(ctx, m->qcur, D, H, 1, 1, m->qcur->nb[1],
                                           m->qcur->nb[2], m->qcur->nb[2], 0);
    const size_t rs = ggml_row_size(GGML_TYPE_F16, D);
    struct ggml_tensor * k_view = ggml_view_4d(ctx, m->kc, D, 1, N, 1, rs, rs, rs * (size_t) N, 0);
    struct ggml_tensor * v_view = ggml_view_4d(ctx, m->kc, R, 1, N, 1, rs, rs, rs * (size_t) N, 0);
    struct ggml_tensor * qp = ggml_permute(ctx, q4, 0, 2, 1, 3);
    struct ggml_tensor * kp = ggml_permute(ctx, k_view, 0, 2, 1, 3);
    struct ggml_tensor * vp = ggml_permute(ctx, v_view, 0, 2, 1, 3);
    struct ggml_tensor * vT = ggml_cont(ctx, ggml_transpose(ctx, vp));
    struct ggml_tensor * kq = ggml_mul_mat(ctx, kp, qp);
    kq = ggml_soft_max_ext(ctx, kq, m->mask, kq_scale, 0.0f);
    m->kqv = ggml_mul_mat(ctx, vT, kq);                                      /* [R, 1, H] */
    /* m1_layer.cpp:502: kqv_mla */
    m->out = ggml_mul_mat(ctx, m->wvb, m->kqv);                              /* [V, 1, H] */

    m->gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(m->gf, m->q_abs);
    ggml_build_forward_expand(m->gf, m->out);

    struct ggml_threadpool_params tpp = ggml_threadpool_params_default(n_threads);
    m->tp = ggml_threadpool_new(&tpp);
    struct ggml_cplan plan = ggml_graph_plan(m->gf, n_threads, m->tp);
    m->work_size = plan.work_size;
    m->work = (uint8_t *) malloc(m->work_size > 0 ? m->work_size : 1);
    return m;
}

ref_mla * ref_mla_create(int H, int nope, int rope, int R, int V, int64_t N, float kq_scale,
                         int n_threads) {
    return ref_mla_create_typed(H, nope, rope, R, V, N, kq_scale, n_threads, GGML_TYPE_F16);
}

void ref_mla_destroy(ref_mla * m) {
    if (!m) return;
    if (m->tp) ggml_threadpool_free(m->tp);
    free(m->work);
    ggml_free(m->ctx);
    free(m);
}

/* Inputs are passed as raw bytes in the ggml layouts listed at the top of this file. */
void ref_mla_set_inputs(ref_mla * m, const float * q, const void * wkb, const uint16_t * kc,
                        const float * mask, const void * wvb) {
    if (q)    memcpy(m->q->data, q, ggml_nbytes(m->q));
    if (wkb)  memcpy(m->wkb->data, wkb, ggml_nbytes(m->wkb));
    if (kc)   memcpy(m->kc->data, kc, ggml_nbytes(m->kc));
    if (mask) memcpy(m->mask->data, mask, ggml_nbytes(m->mask));
    if (wvb)  memcpy(m->wvb->data, wvb, ggml_nbytes(m->wvb));
}

int ref_mla_compute(ref_mla * m) {
    struct ggml_cplan plan = ggml_graph_plan(m->gf, m->n_threads, m->tp);
    if (plan.work_size > m->work_size) return -1;
    plan.work_data = m->work;
    return (int) ggml_graph_compute(m->gf, &plan);
}

/* Taps, copied out: q_abs [H][R], qcur [H][D], attn [H][R], out [H][V] (numpy row-major). */
void ref_mla_get_outputs(const ref_mla * m, float * q_abs, float * qcur, float * attn, float * out) {
    if (q_abs) memcpy(q_abs, m->q_abs->data, ggml_nbytes(m->q_abs));
    if (qcur)  memcpy(qcur, m->qcur->data, ggml_nbytes(m->qcur));
    if (attn)  memcpy(attn, m->kqv->data, ggml_nbytes(m->kqv));
    if (out)   memcpy(out, m->out->data, ggml_nbytes(m->out));
}

int ref_mla_n_nodes(const ref_mla * m) { return ggml_graph_n_nodes(m->gf); }

/* ------------------------------------------------------------------------------------------
 * The unfused KV-write (engine/m1_layer.cpp:422-460, flag OFF), one token.
 *   cur     F32  [n_in, 1]      the attn_norm output
 *   wkv_a   Q8_0 [n_in, D]      D = R + rope (the KV row)
 *   kv_norm F32  [R]
 *   kcache  F16  [D, N]         written in place by set_rows
 *   kidx    I64  [1], pos I32 [1]
 * Taps: Kcur F32 [D] (the normed + roped row, = the values set_rows writes), the cache.
 * ------------------------------------------------------------------------------------------ */
typedef struct ref_kvw {
    int n_in, R, rope, n_threads;
    int64_t N;
    struct ggml_context * ctx;
    struct ggml_cgraph * gf;
    struct ggml_threadpool * tp;
    uint8_t * work;
    size_t work_size;
    struct ggml_tensor *cur, *w, *nw, *kc, *kidx, *pos, *kcur;
} ref_kvw;

ref_kvw * ref_kvw_create(int n_in, int R, int rope, int64_t N, float eps, float freq_base,
                         float freq_scale, float ext_factor, float attn_factor, float beta_fast,
                         float beta_slow, int n_ctx_orig, int n_threads) {
    if (n_in <= 0 || n_in % 32 || R <= 0 || rope <= 0 || N <= 0 || n_threads <= 0) return NULL;
    ref_kvw * m = (ref_kvw *) calloc(1, sizeof(ref_kvw));
    m->n_in = n_in; m->R = R; m->rope = rope; m->N = N; m->n_threads = n_threads;
    const int D = R + rope;
    size_t bytes = (size_t) n_in * 4 + ggml_row_size(GGML_TYPE_Q8_0, n_in) * D + (size_t) R * 4 +
                   (size_t) D * N * 2 + 64 + (size_t) D * 4 * 8 +
                   64 * ggml_tensor_overhead() + ggml_graph_overhead() + (1u << 20);
    struct ggml_init_params ip = { bytes, NULL, false };
    m->ctx = ggml_init(ip);
    if (!m->ctx) { free(m); return NULL; }
    struct ggml_context * ctx = m->ctx;
    m->cur  = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, n_in, 1);
    m->w    = ggml_new_tensor_2d(ctx, GGML_TYPE_Q8_0, n_in, D);
    m->nw   = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, R);
    m->kc   = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, D, N);
    m->kidx = ggml_new_tensor_1d(ctx, GGML_TYPE_I64, 1);
    m->pos  = ggml_new_tensor_1d(ctx, GGML_TYPE_I32, 1);

    /* m1_layer.cpp:424-434 */
    struct ggml_tensor * kv = ggml_mul_mat(ctx, m->w, m->cur);                     /* [D, 1] */
    const size_t rs = ggml_row_size(kv->type, D);
    struct ggml_tensor * kv_cmpr = ggml_view_2d(ctx, kv, R, 1, rs, 0);
    struct ggml_tensor * k_pe = ggml_view_3d(ctx, kv, rope, 1, 1, rs, rs,
                                             ggml_row_size(kv->type, R));
    k_pe = ggml_rope_ext(ctx, k_pe, m->pos, NULL, rope, 0 /* NORMAL */, n_ctx_orig, freq_base,
                         freq_scale, ext_factor, attn_factor, beta_fast, beta_slow);
    kv_cmpr = ggml_mul(ctx, ggml_rms_norm(ctx, kv_cmpr, eps), m->nw);
    /* m1_layer.cpp:452-458: Kcur = concat(kv_cmpr, k_pe), then set_rows into the cache */
    m->kcur = ggml_concat(ctx, ggml_reshape_3d(ctx, kv_cmpr, R, 1, 1), k_pe, 0);   /* [D, 1, 1] */
    struct ggml_tensor * wr = ggml_set_rows(ctx, m->kc, ggml_reshape_2d(ctx, m->kcur, D, 1),
                                            m->kidx);

    m->gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(m->gf, wr);
    ggml_build_forward_expand(m->gf, m->kcur);
    struct ggml_threadpool_params tpp = ggml_threadpool_params_default(n_threads);
    m->tp = ggml_threadpool_new(&tpp);
    struct ggml_cplan plan = ggml_graph_plan(m->gf, n_threads, m->tp);
    m->work_size = plan.work_size;
    m->work = (uint8_t *) malloc(m->work_size > 0 ? m->work_size : 1);
    return m;
}

void ref_kvw_set_inputs(ref_kvw * m, const float * cur, const void * w, const float * nw,
                        const uint16_t * kc, int64_t kidx, int32_t pos) {
    if (cur) memcpy(m->cur->data, cur, ggml_nbytes(m->cur));
    if (w)   memcpy(m->w->data, w, ggml_nbytes(m->w));
    if (nw)  memcpy(m->nw->data, nw, ggml_nbytes(m->nw));
    if (kc)  memcpy(m->kc->data, kc, ggml_nbytes(m->kc));
    memcpy(m->kidx->data, &kidx, sizeof(kidx));
    memcpy(m->pos->data, &pos, sizeof(pos));
}

int ref_kvw_compute(ref_kvw * m) {
    struct ggml_cplan plan = ggml_graph_plan(m->gf, m->n_threads, m->tp);
    if (plan.work_size > m->work_size) return -1;
    plan.work_data = m->work;
    return (int) ggml_graph_compute(m->gf, &plan);
}

void ref_kvw_get_outputs(const ref_kvw * m, float * kcur, uint16_t * kc) {
    if (kcur) memcpy(kcur, m->kcur->data, ggml_nbytes(m->kcur));
    if (kc)   memcpy(kc, m->kc->data, ggml_nbytes(m->kc));
}

void ref_kvw_destroy(ref_kvw * m) {
    if (!m) return;
    if (m->tp) ggml_threadpool_free(m->tp);
    free(m->work);
    ggml_free(m->ctx);
    free(m);
}
