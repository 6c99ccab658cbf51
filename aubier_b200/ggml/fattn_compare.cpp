// fattn_compare.cpp -- times upstream ggml-cuda's FLASH_ATTN_EXT at the MLA decode shape on a B200,
// as a comparator for the fused path (built by fattn.mk; upstream's kernels are measured, not used).
//
// One decode token, 32 heads, K = the 576-wide latent+rope cache rows, V = the first 512 columns of
// the same rows (a view, as llama.cpp's MLA graph builds it, src/models/deepseek2.cpp:549-587),
// f16 cache, f32 query, the causal mask (all cells of the window open), kq_scale = 1/sqrt(192),
// GGML_PREC_F32.  L layers, each with its own cache, in one graph on the CUDA backend; the graph is
// computed `reps` times (ggml-cuda replays it as a CUDA graph) between two synchronisations, and
// the wall time per layer is printed as one JSON line, with the last layer's output checked
// against a double-precision evaluation on the host (max |out - ref| / max |ref|).
//
// usage: fattn_compare N_KEYS LAYERS REPS
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "ggml.h"
#include "ggml-alloc.h"
#include "ggml-backend.h"
#include "ggml-cuda.h"

// Fills t with N(0, 1) values and returns them as the device holds them (f16-rounded for f16).
static std::vector<float> fill_normal(ggml_tensor * t, uint64_t seed) {
    std::mt19937_64 rng(seed);
    std::normal_distribution<float> nd(0.0f, 1.0f);
    const int64_t n = ggml_nelements(t);
    std::vector<float> v((size_t) n);
    if (t->type == GGML_TYPE_F16) {
        std::vector<ggml_fp16_t> h((size_t) n);
        for (size_t i = 0; i < h.size(); ++i) {
            h[i] = ggml_fp32_to_fp16(nd(rng));
            v[i] = ggml_fp16_to_fp32(h[i]);
        }
        ggml_backend_tensor_set(t, h.data(), 0, h.size() * sizeof(ggml_fp16_t));
    } else {
        for (auto & x : v) x = nd(rng);
        ggml_backend_tensor_set(t, v.data(), 0, v.size() * sizeof(float));
    }
    return v;
}

// max |out - ref| / max |ref| against a double-precision evaluation of one layer on the host:
// out[h][j] = sum_n softmax_n(scale * q[h] . k[n]) k[n][j], j < DV (V = the first DV columns of K).
static double check_layer(const std::vector<float> & q, const std::vector<float> & k,
                          const std::vector<float> & out, int64_t N, int H, int DK, int DV,
                          double scale) {
    double max_ref = 0.0, max_err = 0.0;
    std::vector<double> s((size_t) N);
    for (int h = 0; h < H; ++h) {
        const float * qh = q.data() + (size_t) h * DK;
        double m = -INFINITY;
        for (int64_t n = 0; n < N; ++n) {
            const float * kn = k.data() + (size_t) n * DK;
            double d = 0.0;
            for (int c = 0; c < DK; ++c) d += (double) qh[c] * kn[c];
            s[n] = d * scale;
            m = std::max(m, s[n]);
        }
        double l = 0.0;
        for (int64_t n = 0; n < N; ++n) l += (s[n] = std::exp(s[n] - m));
        std::vector<double> o((size_t) DV, 0.0);
        for (int64_t n = 0; n < N; ++n) {
            const float * kn = k.data() + (size_t) n * DK;
            for (int j = 0; j < DV; ++j) o[j] += s[n] * kn[j];
        }
        for (int j = 0; j < DV; ++j) {
            const double r = o[j] / l;
            max_ref = std::max(max_ref, std::fabs(r));
            max_err = std::max(max_err, std::fabs(r - out[(size_t) h * DV + j]));
        }
    }
    return max_err / max_ref;
}

int main(int argc, char ** argv) {
    if (argc < 4) {
        std::fprintf(stderr, "usage: %s N_KEYS LAYERS REPS\n", argv[0]);
        return 2;
    }
    const int64_t N = std::atoll(argv[1]);
    const int L = std::atoi(argv[2]), reps = std::atoi(argv[3]);
    const int H = 32, DK = 576, DV = 512;
    const float scale = 1.0f / std::sqrt(192.0f);

    ggml_backend_t be = ggml_backend_cuda_init(0);
    if (!be) { std::fprintf(stderr, "no CUDA backend\n"); return 1; }

    ggml_init_params ip = {ggml_tensor_overhead() * (size_t) (16 * L + 64) + ggml_graph_overhead(), nullptr, true};
    ggml_context * ctx = ggml_init(ip);
    std::vector<ggml_tensor *> q(L), kc(L), mask(L), out(L);
    const int64_t mask_rows = 1;   // mask [n_kv, n_batch]
    for (int l = 0; l < L; ++l) {
        q[l] = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, DK, 1, H);          // [576, n_tokens, heads]
        kc[l] = ggml_new_tensor_3d(ctx, GGML_TYPE_F16, DK, N, 1);        // [576, n_kv, 1 kv head]
        mask[l] = ggml_new_tensor_2d(ctx, GGML_TYPE_F16, N, mask_rows);
    }
    ggml_cgraph * gf = ggml_new_graph_custom(ctx, 16 * L + 64, false);
    for (int l = 0; l < L; ++l) {
        ggml_tensor * v = ggml_view_3d(ctx, kc[l], DV, N, 1, kc[l]->nb[1], kc[l]->nb[2], 0);
        out[l] = ggml_flash_attn_ext(ctx, q[l], kc[l], v, mask[l], scale, 0.0f, 0.0f);
        ggml_prec_set_acc(out[l], GGML_PREC_F32);
        ggml_build_forward_expand(gf, out[l]);
    }
    ggml_backend_buffer_t buf = ggml_backend_alloc_ctx_tensors(ctx, be);
    if (!buf) { std::fprintf(stderr, "allocation failed\n"); return 1; }
    std::vector<float> q_last, k_last;
    for (int l = 0; l < L; ++l) {
        std::vector<float> qv = fill_normal(q[l], 1000 * l + 1);
        std::vector<float> kv = fill_normal(kc[l], 1000 * l + 2);
        if (l == L - 1) {
            q_last.swap(qv);
            k_last.swap(kv);
        }
        std::vector<ggml_fp16_t> m((size_t) N * mask_rows, ggml_fp32_to_fp16(0.0f));
        ggml_backend_tensor_set(mask[l], m.data(), 0, m.size() * sizeof(ggml_fp16_t));
    }
    if (!ggml_backend_supports_op(be, out[0])) { std::fprintf(stderr, "FLASH_ATTN_EXT unsupported\n"); return 1; }

    for (int i = 0; i < 3; ++i)   // warm-up: the first computes capture the CUDA graph
        if (ggml_backend_graph_compute(be, gf) != GGML_STATUS_SUCCESS) return 1;
    ggml_backend_synchronize(be);
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < reps; ++i) ggml_backend_graph_compute(be, gf);
    ggml_backend_synchronize(be);
    const auto t1 = std::chrono::steady_clock::now();
    const double us = std::chrono::duration<double, std::micro>(t1 - t0).count() / ((double) reps * L);
    const double bytes = (double) N * DK * 2 + (double) DK * H * 4 + (double) DV * H * 4;
    // the last layer's output, [DV, H, 1 token] (the op's permuted layout), against fp64
    std::vector<float> o((size_t) DV * H);
    ggml_backend_tensor_get(out[L - 1], o.data(), 0, o.size() * sizeof(float));
    const double err = check_layer(q_last, k_last, o, N, H, DK, DV, scale);
    std::printf("{\"n_keys\": %lld, \"layers\": %d, \"reps\": %d, \"us_per_layer\": %.3f, "
                "\"gbs\": %.1f, \"rel_err_vs_fp64\": %.3e, \"kernel\": \"ggml-cuda FLASH_ATTN_EXT "
                "(DKQ 576, DV 512, f16 cache, GGML_PREC_F32)\"}\n",
                (long long) N, L, reps, us, bytes / us * 1e-3, err);
    ggml_backend_buffer_free(buf);
    ggml_free(ctx);
    ggml_backend_free(be);
    return 0;
}
