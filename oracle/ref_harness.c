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

/* Build the graph once; inputs are then written with ref_mla_set_* and computed repeatedly. */
ref_mla * ref_mla_create(int H, int nope, int rope, int R, int V, int64_t N, float kq_scale,
                         int n_threads) {
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
    m->wkb  = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, nope, R, H);
    m->kc   = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, D, N);
    m->mask = ggml_new_tensor_4d(ctx, GGML_TYPE_F32, N, 1, 1, 1);
    m->wvb  = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, R, V, H);

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

void ref_mla_destroy(ref_mla * m) {
    if (!m) return;
    if (m->tp) ggml_threadpool_free(m->tp);
    free(m->work);
    ggml_free(m->ctx);
    free(m);
}

/* Inputs are passed as raw bytes in the ggml layouts listed at the top of this file. */
void ref_mla_set_inputs(ref_mla * m, const float * q, const uint16_t * wkb, const uint16_t * kc,
                        const float * mask, const uint16_t * wvb) {
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
