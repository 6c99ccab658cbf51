/*
 * m4b_ggml_check.c -- checks the ggml side of the drop-in boundary on the CPU, against the
 * reference's vendored ggml with m4b-ggml.patch applied (built by aubier_b200/ggml/ggml.mk).
 *
 *   graphs        builds every M4 node of both head geometries through the ggml_m4_* builders
 *                 (Mistral Small 4: Q8_0 weights, KV row 320; f16 weights, KV row 576), the way
 *                 engine/m1_layer.cpp:415-502 builds them (q_nope a view of q with the full q head
 *                 stride, the mask [n_kv, 1]), plus the token-batch and ragged forms; prints one
 *                 line per node: name, ne[0..3], op, and libm4b's supports_op verdict computed as
 *                 ggml-cuda's supports_op computes it (m4-b200.cu), before any memory exists
 *   unsupported   prints supports_op for nodes whose operands were changed after building to
 *                 shapes neither geometry has (expected 0: ggml then keeps the stock ops)
 *   abort:OP      computes a graph holding an M4 node (OP = wkb, kqkv, phase) on the ggml-cpu
 *                 backend: ggml-cpu.c aborts (the ops have no CPU handler, ggml-cpu.c:2064-2082)
 *   assert:CASE   calls a builder with a shape of neither geometry: GGML_ASSERT aborts
 *
 * Exit 0 on success; the abort modes end with SIGABRT.  Driven by tests/test_ggml_boundary.py.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ggml.h"
#include "ggml-cpu.h"
#include "m4b.h"

static m4b_tensor shape_of(const struct ggml_tensor * t) {
    m4b_tensor r;
    memset(&r, 0, sizeof(r));
    if (!t) return r;
    r.data = t->data ? t->data : (void *) (uintptr_t) 256;   /* placeholder before allocation */
    r.type = (int32_t) t->type;
    for (int i = 0; i < 4; ++i) {
        r.ne[i] = t->ne[i];
        r.nb[i] = t->nb[i];
    }
    return r;
}

static int supports(const struct ggml_tensor * op) {
    m4b_tensor srcs[6];
    int n = 0;
    for (; n < 6; ++n) srcs[n] = shape_of(op->src[n]);
    while (n > 0 && op->src[n - 1] == NULL) --n;
    const m4b_tensor d = shape_of(op);
    const int which = op->op == GGML_OP_M4_WKB ? 0 : op->op == GGML_OP_M4_KQKV ? 1 : 2;
    return m4b_supports_op(which, srcs, n, &d, op->op_params);
}

static void report(const char * name, const struct ggml_tensor * t) {
    printf("%s %lld %lld %lld %lld %s %d\n", name, (long long) t->ne[0], (long long) t->ne[1],
           (long long) t->ne[2], (long long) t->ne[3], ggml_op_name(t->op), supports(t));
}

static struct ggml_context * context(int alloc) {
    struct ggml_init_params p = {256u << 20, NULL, alloc ? false : true};
    return ggml_init(p);
}

/* The nodes of one layer in the f16 geometry: WKB over the q_nope view of q [192, 32, T], KQKV
 * over a [576, n_kv] cache with its mask, PHASE selector 1 (W_UV). */
struct layer {
    struct ggml_tensor *wkb, *kqkv, *wvb;
};

static struct layer f16_layer(struct ggml_context * ctx, int64_t n_kv, int T) {
    struct layer L;
    struct ggml_tensor * w_uk = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, 128, 512, 32);
    struct ggml_tensor * q = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 192, 32, T);
    struct ggml_tensor * q_nope = ggml_view_3d(ctx, q, 128, 32, T, q->nb[1], q->nb[2], 0);
    L.wkb = ggml_m4_wkb(ctx, w_uk, q_nope);
    struct ggml_tensor * kc = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, 576, n_kv);
    struct ggml_tensor * qcur = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 576, 32);
    struct ggml_tensor * mask = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, n_kv, 1);
    L.kqkv = ggml_m4_kqkv(ctx, kc, qcur, mask, 0.0721687836f);
    struct ggml_tensor * w_uv = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, 512, 128, 32);
    L.wvb = ggml_m4_phase_wvb(ctx, w_uv, L.kqkv);
    return L;
}

static int mode_graphs(void) {
    struct ggml_context * ctx = context(0);
    /* f16 geometry, one token (the engine's step) */
    struct layer L = f16_layer(ctx, 262144, 1);
    report("f16.wkb", L.wkb);
    report("f16.kqkv", L.kqkv);
    report("f16.wvb", L.wvb);
    /* f16 geometry, a batch of 16 tokens: WKB / WVB over the batch, the ragged KQKV */
    struct ggml_tensor * w_uk = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, 128, 512, 32);
    struct ggml_tensor * qb = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 192, 32, 16);
    struct ggml_tensor * qb_nope = ggml_view_3d(ctx, qb, 128, 32, 16, qb->nb[1], qb->nb[2], 0);
    report("f16.wkb_batch", ggml_m4_wkb(ctx, w_uk, qb_nope));
    struct ggml_tensor * kc = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, 576, 467089);
    struct ggml_tensor * qcb = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 576, 32, 16);
    struct ggml_tensor * base = ggml_new_tensor_1d(ctx, GGML_TYPE_I32, 16);
    struct ggml_tensor * len = ggml_new_tensor_1d(ctx, GGML_TYPE_I32, 16);
    struct ggml_tensor * attn_b = ggml_m4_kqkv_ragged(ctx, kc, qcb, base, len, 0.0721687836f);
    report("f16.kqkv_ragged", attn_b);
    struct ggml_tensor * w_uv = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, 512, 128, 32);
    report("f16.wvb_batch", ggml_m4_phase_wvb(ctx, w_uv, attn_b));

    /* Mistral Small 4 geometry (engine/m1_layer.h:47-55), the reference's own shapes */
    struct ggml_tensor * mw_uk = ggml_new_tensor_3d(ctx, GGML_TYPE_Q8_0, 64, 256, 32);
    struct ggml_tensor * mq = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 128, 32, 1);
    struct ggml_tensor * mq_nope = ggml_view_3d(ctx, mq, 64, 32, 1, mq->nb[1], mq->nb[2], 0);
    report("q8.wkb", ggml_m4_wkb(ctx, mw_uk, mq_nope));
    struct ggml_tensor * mkc = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, 320, 2501);
    struct ggml_tensor * mqcur = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 320, 32);
    struct ggml_tensor * mmask = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 2501, 1);
    struct ggml_tensor * mattn = ggml_m4_kqkv(ctx, mkc, mqcur, mmask, 0.1f);
    report("q8.kqkv", mattn);
    struct ggml_tensor * mw_uv = ggml_new_tensor_3d(ctx, GGML_TYPE_Q8_0, 256, 128, 32);
    report("q8.wvb", ggml_m4_phase_wvb(ctx, mw_uv, mattn));
    struct ggml_tensor * cur = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 4096, 1);
    struct ggml_tensor * wkv = ggml_new_tensor_2d(ctx, GGML_TYPE_Q8_0, 4096, 320);
    struct ggml_tensor * kvn = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, 256);
    struct ggml_tensor * kidx = ggml_new_tensor_1d(ctx, GGML_TYPE_I64, 1);
    struct ggml_tensor * pos = ggml_new_tensor_1d(ctx, GGML_TYPE_I32, 1);
    report("q8.kvwrite", ggml_m4_phase_kvwrite(ctx, cur, wkv, kvn, mkc, kidx, pos, 10000.0f,
                                               0.0078125f, 1.0f, 0.67f, 32.0f, 1.0f, 1e-6f, 64,
                                               8192));
    ggml_free(ctx);
    return 0;
}

static int mode_unsupported(void) {
    struct ggml_context * ctx = context(0);
    struct layer L = f16_layer(ctx, 4096, 1);
    /* each case changes one operand after the builder accepted it, then restores it */
    struct ggml_tensor * mask = L.kqkv->src[2];
    mask->ne[0] = 4095;                       /* mask shorter than the cache */
    report("mask_len", L.kqkv);
    mask->ne[0] = 4096;
    L.kqkv->src[1]->type = GGML_TYPE_F16;     /* an f16 query */
    report("q_type", L.kqkv);
    L.kqkv->src[1]->type = GGML_TYPE_F32;
    L.wkb->src[0]->ne[1] = 256;               /* W_UK of neither geometry */
    report("w_uk_shape", L.wkb);
    L.wkb->src[0]->ne[1] = 512;
    int32_t * params = (int32_t *) L.wvb->op_params;
    params[0] = 7;                            /* an unknown phase selector */
    report("phase_7", L.wvb);
    params[0] = 1;
    report("restored_kqkv", L.kqkv);          /* back to the supported shapes */
    report("restored_wkb", L.wkb);
    report("restored_wvb", L.wvb);
    ggml_free(ctx);
    return 0;
}

static int mode_abort(const char * op) {
    struct ggml_context * ctx = context(1);
    struct layer L = f16_layer(ctx, 256, 1);
    struct ggml_tensor * node = strcmp(op, "wkb") == 0 ? L.wkb : L.kqkv;
    if (strcmp(op, "phase") == 0) {          /* W_UV over a plain input: the only M4 node */
        struct ggml_tensor * x = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 512, 1, 32);
        node = ggml_m4_phase_wvb(ctx, L.wvb->src[0], x);
    }
    struct ggml_cgraph * gf = ggml_new_graph(ctx);
    ggml_build_forward_expand(gf, node);
    fprintf(stderr, "computing %s on the CPU backend\n", ggml_op_name(node->op));
    ggml_graph_compute_with_ctx(ctx, gf, 1);   /* expected to abort */
    fprintf(stderr, "returned: no abort\n");
    ggml_free(ctx);
    return 3;
}

static int mode_assert(const char * which) {
    struct ggml_context * ctx = context(0);
    if (strcmp(which, "wkb") == 0) {          /* f16 W_UK with the Mistral row count */
        struct ggml_tensor * w = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, 128, 256, 32);
        struct ggml_tensor * q = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 128, 32, 1);
        ggml_m4_wkb(ctx, w, q);
    } else if (strcmp(which, "kqkv") == 0) {  /* a KV row of neither geometry */
        struct ggml_tensor * kc = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, 512, 100);
        struct ggml_tensor * q = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 512, 32);
        struct ggml_tensor * m = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, 100, 1);
        ggml_m4_kqkv(ctx, kc, q, m, 0.1f);
    } else {                                  /* W_UV f16 over a 256-wide attention */
        struct ggml_tensor * w = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, 256, 128, 32);
        struct ggml_tensor * x = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, 256, 1, 32);
        ggml_m4_phase_wvb(ctx, w, x);
    }
    fprintf(stderr, "returned: no assert\n");
    ggml_free(ctx);
    return 3;
}

int main(int argc, char ** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: %s graphs | unsupported | abort:OP | assert:CASE\n", argv[0]);
        return 2;
    }
    if (strcmp(argv[1], "graphs") == 0) return mode_graphs();
    if (strcmp(argv[1], "unsupported") == 0) return mode_unsupported();
    if (strncmp(argv[1], "abort:", 6) == 0) return mode_abort(argv[1] + 6);
    if (strncmp(argv[1], "assert:", 7) == 0) return mode_assert(argv[1] + 7);
    return 2;
}
