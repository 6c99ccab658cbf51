/*
 * mla_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the arithmetic the reference's *unfused* CPU ggml graph performs for
 * MLA decode attention (the numerics oracle of jmars/aubier: the flag-OFF op sequence of
 * engine/m1_layer.cpp:443-502, run by the vendored ggml-cpu).  Only tests/, the smoke check in
 * __graft_entry__.py and the CPU-baseline leg of bench.py may load it, and only as the checker.
 * The product path (aubier_b200/) never links, loads or calls it.
 *
 * The rounding points are the reference's, not ours:
 *   - ggml-cpu mul_mat with an F16 src0 converts an F32 src1 to F16 (round to nearest even) before
 *     the dot (vendor/llama.cpp/ggml/src/ggml-cpu/ggml-cpu.c:1330-1375, vec_dot_type of F16 is F16,
 *     ggml-cpu.c:222-227).  So q (in W_UK . q_nope and in K . Qcur), the softmax probabilities P
 *     (in V^T . P) and the attention output (in W_UV . attn) are all rounded to f16 here.
 *   - the dot itself accumulates f16*f16 products; ggml sums them in f32 SIMD lanes
 *     (vec.cpp:264 ggml_vec_dot_f16); this restatement sums the (exact) products in double, which
 *     is the same math with less rounding noise -- the tolerance absorbs the difference.
 *   - soft_max_ext: w = kq*scale, then w += mask (two f32 roundings, ops.cpp:5874-5886), max,
 *     e = exp(w - max) in f32, sum in double, P = e * (float)(1/sum) (ops.cpp:5895-5906,
 *     vec.cpp:531-600).
 *
 * The split-K partial / merge helpers restate the fused reference's online-softmax merge rule
 * (patches/ggml-m4/m4-kqkv.cu:318-338): m_star = max m_i; l_star = sum l_i e^{m_i-m_star};
 * o_star = sum o_i e^{m_i-m_star}; out = o_star / l_star; a head whose every split is fully masked yields 0.
 * Partials here keep m in log2 units (m = max_n s_n*log2(e)), the convention of the CUDA path.
 *
 * Layouts (numpy row-major view of the ggml tensors; ggml ne[] is the reverse of these shapes):
 *   W_UK  f16 [H][R][K]      ggml [K, R, H]      (K = q_nope width, R = latent)
 *   q     f32 [H][q_stride]  ggml [*, H] with nb1 = 4*q_stride (q_nope = first K floats of a head)
 *   kc    f16 [N][D]         ggml [D, N]         (D = K row = latent + rope; V = first R columns)
 *   mask  f32 [N]            ggml [N, 1]
 *   attn  f32 [H][R]         ggml [R, 1, H]
 *   W_UV  f16 [H][V][R]      ggml [R, V, H]
 *   out   f32 [H][V]         ggml [V, 1, H]
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef uint16_t f16_t;

static inline float h2f(f16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float) v;
}

static inline f16_t f2h(float f) {
    _Float16 v = (_Float16) f; /* IEEE round-to-nearest-even, like ggml_compute_fp32_to_fp16 */
    f16_t h;
    memcpy(&h, &v, 2);
    return h;
}

/* f32 -> f16 -> f32, the rounding ggml applies to an F32 src1 of an F16 mul_mat */
static inline float round_f16(float f) { return h2f(f2h(f)); }

void orc_f32_to_f16(const float * x, f16_t * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = f2h(x[i]);
}

void orc_f16_to_f32(const f16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = h2f(x[i]);
}

/* One f16 x f16 dot, products summed in double (see the header note on accumulation order). */
static double dot_f16(const f16_t * a, const float * b16, int n) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double) h2f(a[i]) * (double) b16[i];
    return s;
}

/*
 * WKB: q_abs[h][r] = sum_k W_UK[h][r][k] * f16(q[h][k]).
 * Restates mul_mat(wk_b, permute(q_nope)) (engine/m1_layer.cpp:443-447) on the CPU backend.
 * out_stride is the head stride of the output in floats (R for the contiguous ggml dst).
 */
void orc_wkb_f16(const f16_t * w, const float * q, int64_t q_stride, int H, int R, int K,
                 float * out, int64_t out_stride) {
    float * q16 = (float *) malloc(sizeof(float) * (size_t) K);
    for (int h = 0; h < H; ++h) {
        for (int k = 0; k < K; ++k) q16[k] = round_f16(q[(size_t) h * q_stride + k]);
        for (int r = 0; r < R; ++r) {
            const f16_t * wr = w + ((size_t) h * R + r) * K;
            out[(size_t) h * out_stride + r] = (float) dot_f16(wr, q16, K);
        }
    }
    free(q16);
}

/*
 * KQKV, the unfused way: kq = K . f16(q) -> soft_max_ext(kq, mask, scale) -> V^T . f16(P).
 * Restates m1_layer.cpp:478-494 (mul_mat(kp, qp), soft_max_ext, cont(transpose(V)), mul_mat).
 * q: [H][q_stride] f32 with the D-wide query at the start of each head.
 * A head whose every key is masked produces NaN in ggml (ops.cpp asserts sum > 0); here it
 * produces 0, the fused reference's convention (m4-kqkv.cu:337), so tests can compare.
 */
void orc_kqkv(const f16_t * kc, int64_t N, int D, int R, const float * q, int64_t q_stride,
              int H, const float * mask, float scale, float * out) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int h = 0; h < H; ++h) {
        float * q16 = (float *) malloc(sizeof(float) * (size_t) D);
        float * w   = (float *) malloc(sizeof(float) * (size_t) (N > 0 ? N : 1));
        float * p16 = (float *) malloc(sizeof(float) * (size_t) (N > 0 ? N : 1));
        double * acc = (double *) malloc(sizeof(double) * (size_t) R);
        for (int d = 0; d < D; ++d) q16[d] = round_f16(q[(size_t) h * q_stride + d]);
        float mx = -INFINITY;
        for (int64_t n = 0; n < N; ++n) {
            const float kq = (float) dot_f16(kc + (size_t) n * D, q16, D);
            float v = kq * scale;
            v = v + (mask ? mask[n] : 0.0f);
            w[n] = v;
            if (v > mx) mx = v;
        }
        if (mx == -INFINITY) {
            for (int r = 0; r < R; ++r) out[(size_t) h * R + r] = 0.0f;
            free(q16); free(w); free(p16); free(acc);
            continue;
        }
        double sum = 0.0;
        for (int64_t n = 0; n < N; ++n) {
            const float e = expf(w[n] - mx);
            w[n] = e;
            sum += (double) e;
        }
        const float inv = (float) (1.0 / sum);
        for (int64_t n = 0; n < N; ++n) p16[n] = round_f16(w[n] * inv);
        for (int r = 0; r < R; ++r) acc[r] = 0.0;
        for (int64_t n = 0; n < N; ++n) {
            if (p16[n] == 0.0f) continue;
            const f16_t * v = kc + (size_t) n * D;
            const double p = (double) p16[n];
            for (int r = 0; r < R; ++r) acc[r] += p * (double) h2f(v[r]);
        }
        for (int r = 0; r < R; ++r) out[(size_t) h * R + r] = (float) acc[r];
        free(q16); free(w); free(p16); free(acc);
    }
}

/*
 * W_UV: out[h][j] = sum_r W_UV[h][j][r] * f16(x[h][r]).
 * Restates mul_mat(wv_b, kqv) (m1_layer.cpp:502).  x_stride = head stride of x in floats.
 */
void orc_wvb_f16(const f16_t * w, const float * x, int64_t x_stride, int H, int V, int R,
                 float * out) {
    float * x16 = (float *) malloc(sizeof(float) * (size_t) R);
    for (int h = 0; h < H; ++h) {
        for (int r = 0; r < R; ++r) x16[r] = round_f16(x[(size_t) h * x_stride + r]);
        for (int j = 0; j < V; ++j)
            out[(size_t) h * V + j] = (float) dot_f16(w + ((size_t) h * V + j) * R, x16, R);
    }
    free(x16);
}

/*
 * Split-K partial over keys [k0, k1): per head, m (log2 units), l and o[R], unnormalised:
 *   s_n = (kq_n*scale + mask_n) * log2(e);  m = max s_n;  l = sum 2^(s_n - m);
 *   o[r] = sum 2^(s_n - m) * V[n][r].
 * Exact (double) -- this checks the partial FORMAT and the merge, not the kernel's roundings.
 * part layout: [H][R + 4] floats: {o[0..R), m, l, 0, 0} (the CUDA path's 16-byte-aligned record).
 */
void orc_kqkv_partial(const f16_t * kc, int64_t k0, int64_t k1, int D, int R, const float * q,
                      int64_t q_stride, int H, const float * mask, float scale, float * part) {
    const double LOG2E = 1.4426950408889634;
    float * q16 = (float *) malloc(sizeof(float) * (size_t) D);
    int64_t n_keys = k1 > k0 ? k1 - k0 : 0;
    double * s = (double *) malloc(sizeof(double) * (size_t) (n_keys > 0 ? n_keys : 1));
    double * acc = (double *) malloc(sizeof(double) * (size_t) R);
    for (int h = 0; h < H; ++h) {
        float * ph = part + (size_t) h * (R + 4);
        for (int d = 0; d < D; ++d) q16[d] = round_f16(q[(size_t) h * q_stride + d]);
        double mx = -INFINITY;
        for (int64_t i = 0; i < n_keys; ++i) {
            const int64_t n = k0 + i;
            const float kq = (float) dot_f16(kc + (size_t) n * D, q16, D);
            const double v = ((double) (kq * scale) + (mask ? (double) mask[n] : 0.0)) * LOG2E;
            s[i] = v;
            if (v > mx) mx = v;
        }
        for (int r = 0; r < R; ++r) acc[r] = 0.0;
        double l = 0.0;
        if (mx > -INFINITY) {
            for (int64_t i = 0; i < n_keys; ++i) {
                if (s[i] == -INFINITY) continue;
                const double e = exp2(s[i] - mx);
                l += e;
                const f16_t * v = kc + (size_t) (k0 + i) * D;
                for (int r = 0; r < R; ++r) acc[r] += e * (double) h2f(v[r]);
            }
        }
        for (int r = 0; r < R; ++r) ph[r] = (float) acc[r];
        ph[R] = (float) mx;
        ph[R + 1] = (float) l;
        ph[R + 2] = 0.0f;
        ph[R + 3] = 0.0f;
    }
    free(q16); free(s); free(acc);
}

/*
 * Merge S partials per head with the online-softmax rule (m4-kqkv.cu:318-338), log2 units.
 * part layout: [S][H][R + 4] records {o[R], m, l, pad, pad}.  out: [H][R] normalised attention
 * (0 for an all-masked head).
 */
void orc_combine(const float * part, int S, int H, int R, float * out) {
    for (int h = 0; h < H; ++h) {
        double mstar = -INFINITY;
        for (int s = 0; s < S; ++s) {
            const double m = part[((size_t) s * H + h) * (R + 4) + R];
            if (m > mstar) mstar = m;
        }
        float * oh = out + (size_t) h * R;
        if (mstar == -INFINITY) {
            for (int r = 0; r < R; ++r) oh[r] = 0.0f;
            continue;
        }
        double lstar = 0.0;
        for (int r = 0; r < R; ++r) oh[r] = 0.0f;
        double * acc = (double *) calloc((size_t) R, sizeof(double));
        for (int s = 0; s < S; ++s) {
            const float * ps = part + ((size_t) s * H + h) * (R + 4);
            if (!(ps[R] > -INFINITY)) continue;
            const double a = exp2((double) ps[R] - mstar);
            lstar += (double) ps[R + 1] * a;
            for (int r = 0; r < R; ++r) acc[r] += (double) ps[r] * a;
        }
        for (int r = 0; r < R; ++r) oh[r] = (float) (acc[r] / lstar);
        free(acc);
    }
}

/*
 * Float64 "exact" attention (no f16 rounding of q or P): a diagnostic reference, used by the
 * full-size property tests where the f16-rounded oracle's own subnormal-P noise dominates.
 */
void orc_kqkv_exact(const f16_t * kc, int64_t N, int D, int R, const float * q, int64_t q_stride,
                    int H, const float * mask, float scale, float * out) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int h = 0; h < H; ++h) {
        double * w = (double *) malloc(sizeof(double) * (size_t) (N > 0 ? N : 1));
        double * acc = (double *) malloc(sizeof(double) * (size_t) R);
        const float * qh = q + (size_t) h * q_stride;
        double mx = -INFINITY;
        for (int64_t n = 0; n < N; ++n) {
            double s = 0.0;
            const f16_t * k = kc + (size_t) n * D;
            for (int d = 0; d < D; ++d) s += (double) h2f(k[d]) * (double) qh[d];
            s = s * (double) scale + (mask ? (double) mask[n] : 0.0);
            w[n] = s;
            if (s > mx) mx = s;
        }
        for (int r = 0; r < R; ++r) acc[r] = 0.0;
        if (mx == -INFINITY) {
            for (int r = 0; r < R; ++r) out[(size_t) h * R + r] = 0.0f;
            free(w); free(acc);
            continue;
        }
        double sum = 0.0;
        for (int64_t n = 0; n < N; ++n) {
            if (w[n] == -INFINITY) continue;
            const double e = exp(w[n] - mx);
            sum += e;
            const f16_t * v = kc + (size_t) n * D;
            for (int r = 0; r < R; ++r) acc[r] += e * (double) h2f(v[r]);
        }
        for (int r = 0; r < R; ++r) out[(size_t) h * R + r] = (float) (acc[r] / sum);
        free(w); free(acc);
    }
}
