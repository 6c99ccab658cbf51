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

/* ============================================================================================
 * The Mistral-Small-4 geometry (engine/m1_layer.h:47-55): Q8_0 weights, Q8 activations.
 *
 * ggml's Q8_0 block (ggml-common.h): an f16 scale d, then 32 int8 quants; value = d * q.
 * Two activation quantizations matter:
 *   CPU graph (the oracle): ggml-cpu's x86 quantize_row_q8_0 with AVX2 / AVX-512 (the build in
 *     oracle/_ref): per 32 values amax; d = amax/127 stored as f16; multiplier 127/amax (0 for
 *     an all-zero block); q = round-half-to-even(x * multiplier)
 *     (ggml-cpu/arch/x86/quants.c:302-346).  The dot is sum_b f16(d_w) f16(d_x) sum_i q_w q_x
 *     (vec_dot_q8_0_q8_0); summed here in double.
 *   Fused reference kernels (MMVQ's Q8_1 form, the numerics GGML_OP_M4_* replicate): per 32
 *     values amax; d = amax/127; the quants round half away from zero, either x / d
 *     (m4-wkb.cu:36-47) or x * (1/d) (m4-phase.cu:69-74 and :107-116); the scale enters the dot
 *     as f16(d).  Restated here with the association of those kernels, in float.
 * ============================================================================================ */
typedef struct {
    f16_t d;
    int8_t qs[32];
} q8_block;   /* 34 bytes, the ggml layout */

/* Weights: quantize rows of K floats (K % 32 == 0) to Q8_0 bytes with ggml's reference
 * quantizer (scale amax/127, multiplier 1/d, roundf; ggml-quants.c quantize_row_q8_0_ref).
 * Only used to make test weights; both sides of a comparison then read the same bytes. */
void orc_q8_0_quantize(const float * x, int64_t rows, int K, uint8_t * out) {
    const int nb = K / 32;
    for (int64_t r = 0; r < rows; ++r) {
        for (int b = 0; b < nb; ++b) {
            const float * xb = x + (size_t) r * K + (size_t) b * 32;
            q8_block blk;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(xb[i]));
            const float d = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            blk.d = f2h(d);
            for (int i = 0; i < 32; ++i) blk.qs[i] = (int8_t) roundf(xb[i] * id);
            memcpy(out + ((size_t) r * nb + b) * 34, &blk, 34);
        }
    }
}

/* Activation block quantizers: q[32] and the f16-rounded scale the dot uses. */
static void quant_cpu(const float * x, int8_t * q, float * d16) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    *d16 = round_f16(amax / 127.0f);
    const float mul = amax != 0.0f ? 127.0f / amax : 0.0f;
    for (int i = 0; i < 32; ++i) q[i] = (int8_t) (int) nearbyintf(x[i] * mul);  /* ties to even */
}

/* mode 0: x / d (m4-wkb.cu), mode 1: x * (1/d) (m4-phase.cu) -- both round half away from zero */
static void quant_fused(const float * x, int8_t * q, float * d16, int mode) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[i]));
    const float d = amax / 127.0f;
    *d16 = round_f16(d);
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int i = 0; i < 32; ++i) {
        float v;
        if (mode == 0) v = amax == 0.0f ? 0.0f : roundf(x[i] / d);
        else v = roundf(x[i] * id);
        q[i] = (int8_t) (int) v;
    }
}

static inline const q8_block * q8_row(const uint8_t * w, int64_t row, int K) {
    return (const q8_block *) (w + (size_t) row * (K / 32) * 34);
}

static inline int dot_i8(const int8_t * a, const int8_t * b) {
    int s = 0;
    for (int i = 0; i < 32; ++i) s += (int) a[i] * (int) b[i];
    return s;
}

/*
 * WKB with Q8_0 W_UK [H][R][K] (ggml [K, R, H]): out[h][r] = W_UK[h][r] . Q8(q[h][0:K]).
 * numerics 0 = the CPU graph (mul_mat Q8_0, m1_layer.cpp:445); 1 = the fused reference kernel
 * (m4-wkb.cu:21-53: acc over the blocks in order, acc += (d_w * f16(d_x)) * sum).
 */
void orc_wkb_q8(const uint8_t * w, const float * q, int64_t q_stride, int H, int R, int K,
                float * out, int64_t out_stride, int numerics) {
    const int nb = K / 32;
    int8_t * xq = (int8_t *) malloc((size_t) K);
    float * xd = (float *) malloc(sizeof(float) * (size_t) nb);
    for (int h = 0; h < H; ++h) {
        for (int b = 0; b < nb; ++b) {
            const float * xb = q + (size_t) h * q_stride + (size_t) b * 32;
            if (numerics == 0) quant_cpu(xb, xq + b * 32, xd + b);
            else quant_fused(xb, xq + b * 32, xd + b, 0);
        }
        for (int r = 0; r < R; ++r) {
            const q8_block * wr = q8_row(w, (int64_t) h * R + r, K);
            if (numerics == 0) {
                double acc = 0.0;
                for (int b = 0; b < nb; ++b)
                    acc += (double) (h2f(wr[b].d) * xd[b]) * (double) dot_i8(wr[b].qs, xq + b * 32);
                out[(size_t) h * out_stride + r] = (float) acc;
            } else {
                float acc = 0.0f;
                for (int b = 0; b < nb; ++b)
                    acc += h2f(wr[b].d) * xd[b] * (float) dot_i8(wr[b].qs, xq + b * 32);
                out[(size_t) h * out_stride + r] = acc;
            }
        }
    }
    free(xq);
    free(xd);
}

/*
 * W_UV with Q8_0 W_UV [H][V][R] (ggml [R, V, H]): out[h][j] = W_UV[h][j] . Q8(x[h][0:R]).
 * numerics 0 = the CPU graph (mul_mat, m1_layer.cpp:502); 1 = the fused reference kernel
 * (m4-phase.cu:52-89: lane l of a warp owns element l of every block, accumulates
 * (d_w * f16(d_x)) * (q_w q_x) over the blocks, then a butterfly sum over the 32 lanes).
 */
void orc_wvb_q8(const uint8_t * w, const float * x, int64_t x_stride, int H, int V, int R,
                float * out, int numerics) {
    const int nb = R / 32;
    int8_t * xq = (int8_t *) malloc((size_t) R);
    float * xd = (float *) malloc(sizeof(float) * (size_t) nb);
    for (int h = 0; h < H; ++h) {
        for (int b = 0; b < nb; ++b) {
            const float * xb = x + (size_t) h * x_stride + (size_t) b * 32;
            if (numerics == 0) quant_cpu(xb, xq + b * 32, xd + b);
            else quant_fused(xb, xq + b * 32, xd + b, 1);
        }
        for (int j = 0; j < V; ++j) {
            const q8_block * wr = q8_row(w, (int64_t) h * V + j, R);
            if (numerics == 0) {
                double acc = 0.0;
                for (int b = 0; b < nb; ++b)
                    acc += (double) (h2f(wr[b].d) * xd[b]) * (double) dot_i8(wr[b].qs, xq + b * 32);
                out[(size_t) h * V + j] = (float) acc;
            } else {
                float lane[32];
                for (int l = 0; l < 32; ++l) {
                    float a = 0.0f;
                    for (int b = 0; b < nb; ++b)
                        a += h2f(wr[b].d) * xd[b] *
                             (float) ((int) wr[b].qs[l] * (int) xq[b * 32 + l]);
                    lane[l] = a;
                }
                for (int off = 16; off > 0; off >>= 1) {
                    float nx[32];
                    for (int l = 0; l < 32; ++l) nx[l] = lane[l] + lane[l ^ off];
                    memcpy(lane, nx, sizeof(lane));
                }
                out[(size_t) h * V + j] = lane[0];
            }
        }
    }
    free(xq);
    free(xd);
}

/*
 * YaRN correction dims (the published YaRN rule as ggml applies it, ggml.c:4630-4644): the
 * rotary dims whose wavelength at the original context sits between beta_fast and beta_slow
 * rotations: corr(b) = n_dims * ln(n_ctx_orig / (b * 2 pi)) / (2 ln(base)); the ramp runs from
 * max(0, floor(corr(beta_fast))) to min(n_dims - 1, ceil(corr(beta_slow))).
 */
void orc_rope_corr_dims(int n_dims, int n_ctx_orig, float freq_base, float beta_fast,
                        float beta_slow, float * dims) {
    const float pi = 3.14159265358979323846f;
    const float a = n_dims * logf(n_ctx_orig / (beta_fast * 2 * pi)) / (2 * logf(freq_base));
    const float b = n_dims * logf(n_ctx_orig / (beta_slow * 2 * pi)) / (2 * logf(freq_base));
    dims[0] = fmaxf(0.0f, floorf(a));
    dims[1] = fminf((float) (n_dims - 1), ceilf(b));
}

/* one YaRN-scaled rotation angle and magnitude (ggml-cpu/ops.cpp:6179-6201 rope_yarn) */
static void yarn_cos_sin(float theta_extrap, float freq_scale, const float * corr, int p,
                         float ext_factor, float mscale, float * c, float * s) {
    float theta = freq_scale * theta_extrap;
    if (ext_factor != 0.0f) {
        const float y = ((float) p - corr[0]) / fmaxf(0.001f, corr[1] - corr[0]);
        const float mix = (1.0f - fminf(1.0f, fmaxf(0.0f, y))) * ext_factor;
        theta = theta * (1.0f - mix) + theta_extrap * mix;
        mscale *= 1.0f + 0.1f * logf(1.0f / freq_scale);
    }
    *c = cosf(theta) * mscale;
    *s = sinf(theta) * mscale;
}

/*
 * KV-write for one token (GGML_OP_M4_PHASE selector 0; the flag-OFF sequence of
 * m1_layer.cpp:422-460): kv = W_kva . Q8(cur) [D = R + rope]; Kcur[0:R) = rms_norm(kv[0:R]) *
 * norm_w; Kcur[R:D) = rope_yarn(kv[R:D], pos) in NORMAL mode (pairs (2p, 2p+1)); the cache row
 * kidx receives f16(Kcur).
 * numerics 0 = the CPU graph: Q8_0 activations as quant_cpu, the norm's sum of squares in
 *   double (ops.cpp:4140-4147), the angle pos * theta_scale^p built by repeated multiplication
 *   (ops.cpp:6203-6217);
 * numerics 1 = the fused reference (m4-phase.cu:97-200): Q8_1 activations (x * 1/d), the sum of
 *   squares in float over 10 warp partials then summed in order, the angle pos * powf(theta_scale, p).
 * kcache: [N][D] f16, written at row kidx.  kcur: [D] f32 out.
 */
void orc_kvwrite(const float * cur, int n_in, const uint8_t * w, const float * norm_w, int R,
                 int rope, f16_t * kcache, int64_t kidx, int pos, float eps, float freq_base,
                 float freq_scale, float ext_factor, float attn_factor, float beta_fast,
                 float beta_slow, int n_ctx_orig, int numerics, float * kcur) {
    const int D = R + rope;
    const int nb = n_in / 32;
    int8_t * xq = (int8_t *) malloc((size_t) n_in);
    float * xd = (float *) malloc(sizeof(float) * (size_t) nb);
    for (int b = 0; b < nb; ++b) {
        if (numerics == 0) quant_cpu(cur + (size_t) b * 32, xq + b * 32, xd + b);
        else quant_fused(cur + (size_t) b * 32, xq + b * 32, xd + b, 1);
    }
    float * kv = (float *) malloc(sizeof(float) * (size_t) D);
    for (int o = 0; o < D; ++o) {
        const q8_block * wr = q8_row(w, o, n_in);
        double acc = 0.0;
        for (int b = 0; b < nb; ++b)
            acc += (double) (h2f(wr[b].d) * xd[b]) * (double) dot_i8(wr[b].qs, xq + b * 32);
        kv[o] = (float) acc;
    }
    /* RMS norm of [0, R) times the norm weight */
    float scale;
    if (numerics == 0) {
        double ss = 0.0;
        for (int i = 0; i < R; ++i) ss += (double) (kv[i] * kv[i]);
        const float mean = (float) (ss / R);
        scale = 1.0f / sqrtf(mean + eps);
    } else {
        float part[32] = {0};
        const int nw = (D + 31) / 32;
        for (int i = 0; i < R; ++i) part[i / 32] += kv[i] * kv[i];
        float ssf = 0.0f;
        for (int i = 0; i < nw; ++i) ssf += part[i];
        scale = 1.0f / sqrtf(ssf / (float) R + eps);
    }
    for (int i = 0; i < R; ++i) kcur[i] = numerics == 0 ? (kv[i] * scale) * norm_w[i]
                                                        : scale * kv[i] * norm_w[i];
    /* rope of [R, D) */
    float corr[2];
    orc_rope_corr_dims(rope, n_ctx_orig, freq_base, beta_fast, beta_slow, corr);
    const float theta_scale = powf(freq_base, -2.0f / (float) rope);
    float theta_it = (float) pos;
    for (int p = 0; p < rope / 2; ++p) {
        const float te = numerics == 0 ? theta_it : (float) pos * powf(theta_scale, (float) p);
        float c, s;
        yarn_cos_sin(te, freq_scale, corr, p, ext_factor, attn_factor, &c, &s);
        const float x0 = kv[R + 2 * p], x1 = kv[R + 2 * p + 1];
        kcur[R + 2 * p] = x0 * c - x1 * s;
        kcur[R + 2 * p + 1] = x0 * s + x1 * c;
        theta_it *= theta_scale;
    }
    if (kcache)
        for (int i = 0; i < D; ++i) kcache[(size_t) kidx * D + i] = f2h(kcur[i]);
    free(xq);
    free(xd);
    free(kv);
}
