// m4-b200.cu -- ggml-cuda launchers of the M4 ops, as shims over libm4b's C ABI (include/m4b.h).
//
// Goes into ggml/src/ggml-cuda/ of the reference's vendored ggml in place of
// patches/ggml-m4/m4-{wkb,kqkv,phase}.cu, together with m4b-ggml.patch (builders for both head
// geometries and the ragged KQKV, the dispatch include and supports_op).  Built by ggml-cuda's
// own CMake as one more .cu file; link libm4b.so.  Per launch: copy dst->src[i] and dst into the
// ABI's POD structs (data, type, ne[], nb[] -- the m4b_type values are ggml_type ids), take the
// op's scratch from the backend's memory pool (no cudaMalloc inside a captured graph), launch on
// ctx.stream(), and turn a nonzero status into GGML_ABORT, as the reference's launchers assert
// their contract (m4-kqkv.cu:345-355).
#include "m4-b200.cuh"

#include <cstring>

#include "m4b.h"

namespace {

m4b_tensor to_m4b(const ggml_tensor * t) {
    m4b_tensor r;
    std::memset(&r, 0, sizeof(r));
    if (t == nullptr) return r;
    r.data = t->data;
    r.type = static_cast<int32_t>(t->type);
    for (int i = 0; i < 4; ++i) {
        r.ne[i] = t->ne[i];
        r.nb[i] = t->nb[i];
    }
    return r;
}

// supports_op runs while the scheduler assigns backends, before tensors have memory: a present
// operand without data gets a 256-byte-aligned placeholder (never dereferenced) so that it is not
// taken for an absent optional one.
m4b_tensor to_m4b_shape(const ggml_tensor * t) {
    m4b_tensor r = to_m4b(t);
    if (t != nullptr && r.data == nullptr) r.data = reinterpret_cast<void *>(uintptr_t(256));
    return r;
}

void check(int rc, const char * what) {
    if (rc != M4B_OK) {
        const char * cuda = "";
        if (rc == M4B_ECUDA) m4b_last_cuda_error(&cuda);
        GGML_ABORT("%s: %s %s", what, m4b_strerror(rc), cuda ? cuda : "");
    }
}

m4b_stream_t stream_of(ggml_backend_cuda_context & ctx) {
    return reinterpret_cast<m4b_stream_t>(ctx.stream());
}

}  // namespace

void ggml_cuda_m4_wkb(ggml_backend_cuda_context & ctx, ggml_tensor * dst) {
    m4b_wkb_args a;
    std::memset(&a, 0, sizeof(a));
    a.src0 = to_m4b(dst->src[0]);
    a.src1 = to_m4b(dst->src[1]);
    a.dst = to_m4b(dst);
    check(m4b_wkb(&a, stream_of(ctx)), "GGML_OP_M4_WKB");
}

void ggml_cuda_m4_kqkv(ggml_backend_cuda_context & ctx, ggml_tensor * dst) {
    float kq_scale;
    std::memcpy(&kq_scale, dst->op_params, sizeof(float));
    if (dst->src[3] != nullptr) {   // ggml_m4_kqkv_ragged: per-token windows in src[3] / src[4]
        m4b_kqkv_ragged_args a;
        std::memset(&a, 0, sizeof(a));
        a.kcache = to_m4b(dst->src[0]);
        a.q = to_m4b(dst->src[1]);
        a.seq_base = to_m4b(dst->src[3]);
        a.seq_len = to_m4b(dst->src[4]);
        a.dst = to_m4b(dst);
        a.kq_scale = kq_scale;
        const size_t need = m4b_kqkv_ragged_scratch_bytes(dst->src[1]->ne[2]);
        ggml_cuda_pool_alloc<char> scratch(ctx.pool(), need);
        a.scratch = scratch.get();
        a.scratch_bytes = need;
        check(m4b_kqkv_ragged(&a, stream_of(ctx)), "GGML_OP_M4_KQKV (ragged)");
        return;
    }
    m4b_kqkv_args a;
    std::memset(&a, 0, sizeof(a));
    a.src0 = to_m4b(dst->src[0]);
    a.src1 = to_m4b(dst->src[1]);
    a.src2 = to_m4b(dst->src[2]);
    a.dst = to_m4b(dst);
    a.kq_scale = kq_scale;
    const int geometry = dst->src[0]->ne[0] == 320 ? 1 : 0;   // KV row 320: Mistral Small 4
    const size_t need = m4b_kqkv_scratch_bytes(geometry, dst->src[0]->ne[1]);
    ggml_cuda_pool_alloc<char> scratch(ctx.pool(), need);
    a.scratch = scratch.get();
    a.scratch_bytes = need;
    check(m4b_kqkv(&a, stream_of(ctx)), "GGML_OP_M4_KQKV");
}

void ggml_cuda_m4_phase(ggml_backend_cuda_context & ctx, ggml_tensor * dst) {
    m4b_phase_args a;
    std::memset(&a, 0, sizeof(a));
    for (int i = 0; i < 6; ++i) a.src[i] = to_m4b(dst->src[i]);
    a.dst = to_m4b(dst);
    std::memcpy(a.op_params, dst->op_params, sizeof(int32_t) * 10);   // ggml.c:3464-3468
    const size_t need = m4b_phase_scratch_bytes(a.op_params[0]);
    ggml_cuda_pool_alloc<char> scratch(ctx.pool(), need > 0 ? need : 16);
    a.scratch = scratch.get();
    a.scratch_bytes = need;
    check(m4b_phase(&a, stream_of(ctx)), "GGML_OP_M4_PHASE");
}

bool ggml_cuda_m4_supports_op(const ggml_tensor * op) {
    m4b_tensor srcs[6];
    int n = 0;
    for (; n < 6; ++n) srcs[n] = to_m4b_shape(op->src[n]);
    while (n > 0 && op->src[n - 1] == nullptr) --n;   // trailing absent operands
    const m4b_tensor d = to_m4b_shape(op);
    const int which = op->op == GGML_OP_M4_WKB ? 0 : op->op == GGML_OP_M4_KQKV ? 1 : 2;
    return m4b_supports_op(which, srcs, n, &d, op->op_params) != 0;
}
