// m4b_api.cu -- the C ABI (include/m4b.h): contract validation, dispatch and sizes.
//
// Validation mirrors the reference's builders + launchers (vendor/llama.cpp/ggml/src/ggml.c:
// 3398-3540, patches/ggml-m4/m4-*.cu launchers) and supports_op (ggml-cuda.cu:5848-5885), for
// both head geometries; the geometry is read from the operands' shapes and types (the reference
// pins the Mistral-Small-4 one, engine/m1_layer.h:47-55).  Every check runs before any CUDA call;
// a violation launches nothing.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "m4b_internal.h"

namespace m4b {
namespace {

// The two geometries: 0 = BASELINE (f16 weights), 1 = MISTRAL_SMALL (Q8_0 weights).
struct Geom {
    int latent;   // R: kv_lora_rank, the V width
    int krow;     // R + rope: the KV row
    int nope;     // q_nope width
    int part;     // partial record floats: R + 4
};
constexpr Geom kGeo[2] = {{kLatent, kKRow, kNope, kPartStride}, {256, 320, 64, 260}};
constexpr int kGeomBaseline = 0;
constexpr int kGeomMistral = 1;
constexpr int kQ8Block = 34;   // ggml block_q8_0: f16 scale + 32 int8
constexpr int kKvwIn = 4096;   // the KV-write's input width (attn_norm output, m4-phase.cu:21)

bool type_ne(const m4b_tensor& t, int type, int64_t n0, int64_t n1, int64_t n2, int64_t n3) {
    return t.type == type && t.ne[0] == n0 && t.ne[1] == n1 && t.ne[2] == n2 && t.ne[3] == n3;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Contiguous in dims 0..1 / 0..2 (element stride = type size, rows packed).
bool packed3(const m4b_tensor& t, uint64_t esz) {
    return t.nb[0] == esz && t.nb[1] == esz * static_cast<uint64_t>(t.ne[0]) &&
           t.nb[2] == t.nb[1] * static_cast<uint64_t>(t.ne[1]);
}

// A packed Q8_0 tensor [K, rows, heads]: rows of K / 32 blocks.
bool packed_q8(const m4b_tensor& t) {
    const uint64_t row = static_cast<uint64_t>(t.ne[0] / 32) * kQ8Block;
    return t.ne[0] % 32 == 0 && t.nb[0] == kQ8Block && t.nb[1] == row &&
           t.nb[2] == row * static_cast<uint64_t>(t.ne[1]);
}

// Per-device facts, cached (one process may drive several devices).
struct DevInfo {
    int checked = 0;
    int ok = 0;
    int sms = 0;
};
DevInfo g_dev[64];

int device_check(int* sms_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return M4B_ECUDA;
    if (dev < 0 || dev >= 64) return M4B_EDEVICE;
    DevInfo& d = g_dev[dev];
    if (!d.checked) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return M4B_ECUDA;
        d.ok = (major == 10 && minor == 0);
        d.sms = sms;
        d.checked = 1;
    }
    if (!d.ok) return M4B_EDEVICE;
    if (sms_out) *sms_out = d.sms;
    return M4B_OK;
}

int n_tiles(int64_t n_kv) { return static_cast<int>((n_kv + kTileKeys - 1) / kTileKeys); }

int default_splits(int64_t n_kv, int sms) {
    const int cap = sms < kMaxSplits ? sms : kMaxSplits;
    const int t = n_tiles(n_kv);
    return t < cap ? t : cap;
}

int status_of(cudaError_t e) { return e == cudaSuccess ? M4B_OK : M4B_ECUDA; }

// F32 activations [n0, n1, n2] with unit inner stride and 4-byte strides.
bool f32_view(const m4b_tensor& t, int64_t n0, int64_t n1, int64_t n2) {
    return type_ne(t, M4B_TYPE_F32, n0, n1, n2, 1) && t.nb[0] == 4 && t.nb[1] % 4 == 0 &&
           t.nb[2] % 4 == 0 && t.data != nullptr && aligned(t.data, 4);
}

// ---------------------------------------------------------------------------------------------
// WKB.  src0 W_UK: F16 [128, 512, 32] or Q8_0 [64, 256, 32] (m4-wkb.cu:75-81); src1 q_nope
// F32 [nope, 32, T]; dst F32 [R, 32, T].  T = 1 in the reference's op (ggml.c:3398-3423); up to
// kMaxSeqs here, for the ragged batch (token stride nb[2]).
// ---------------------------------------------------------------------------------------------
int check_wkb(const m4b_tensor& w, const m4b_tensor& x, const m4b_tensor& dst, int* geom) {
    int g;
    if (type_ne(w, M4B_TYPE_Q8_0, 64, 256, kHeads, 1)) {
        if (!packed_q8(w) || !w.data || !aligned(w.data, 4)) return M4B_EINVAL;
        g = kGeomMistral;
    } else if (type_ne(w, M4B_TYPE_F16, kNope, kLatent, kHeads, 1)) {
        if (!packed3(w, 2) || !w.data || !aligned(w.data, 16)) return M4B_EINVAL;
        g = kGeomBaseline;
    } else {
        return M4B_EINVAL;
    }
    const Geom& G = kGeo[g];
    const int64_t nt = x.ne[2];
    if (nt < 1 || nt > kMaxSeqs) return M4B_EINVAL;
    if (!f32_view(x, G.nope, kHeads, nt) || x.nb[1] < 4u * G.nope) return M4B_EINVAL;
    if (!f32_view(dst, G.latent, kHeads, nt) || dst.nb[1] < 4u * G.latent) return M4B_EINVAL;
    *geom = g;
    return M4B_OK;
}

// ---------------------------------------------------------------------------------------------
// KQKV.  src0 kcache F16 [576 | 320, N]; src1 q F32 [krow, 32]; src2 mask F32 [N] (optional);
// dst F32 [R, 1, 32] (m4-kqkv.cu:345-355, with the head geometry read from the cache row).
// ---------------------------------------------------------------------------------------------
int kqkv_geometry(const m4b_tensor& kc) {
    if (kc.type != M4B_TYPE_F16) return -1;
    if (kc.ne[0] == kKRow) return kGeomBaseline;
    if (kc.ne[0] == 320) return kGeomMistral;
    return -1;
}

int check_kqkv_inputs(const m4b_kqkv_args& a, int* geom) {
    const m4b_tensor& kc = a.src0;
    const m4b_tensor& q = a.src1;
    const m4b_tensor& mask = a.src2;
    const int g = kqkv_geometry(kc);
    if (g < 0) return M4B_EINVAL;
    const Geom& G = kGeo[g];
    if (kc.ne[1] < 1 || kc.ne[2] != 1 || kc.ne[3] != 1 || kc.nb[0] != 2 || kc.nb[1] % 16 != 0 ||
        kc.nb[1] < 2u * G.krow)
        return M4B_EINVAL;
    if (kc.ne[1] > (int64_t(1) << 30)) return M4B_EINVAL;
    if (!type_ne(q, M4B_TYPE_F32, G.krow, kHeads, 1, 1) || q.nb[0] != 4 || q.nb[1] % 4 != 0 ||
        q.nb[1] < 4u * G.krow)
        return M4B_EINVAL;
    if (mask.data != nullptr) {   // ggml_m4_kqkv: mask ne0 == n_kv, one row
        if (mask.type != M4B_TYPE_F32 || mask.ne[0] != kc.ne[1] || mask.ne[1] != 1 ||
            mask.ne[2] != 1 || mask.ne[3] != 1 || mask.nb[0] != 4 || !aligned(mask.data, 4))
            return M4B_EINVAL;
    }
    if (!kc.data || !q.data || !aligned(kc.data, 16) || !aligned(q.data, 4)) return M4B_EINVAL;
    if (!(a.kq_scale == a.kq_scale)) return M4B_EINVAL;   // NaN scale
    *geom = g;
    return M4B_OK;
}

int check_kqkv(const m4b_kqkv_args& a, int* geom) {
    int rc = check_kqkv_inputs(a, geom);
    if (rc != M4B_OK) return rc;
    const m4b_tensor& d = a.dst;
    const int R = kGeo[*geom].latent;
    if (!type_ne(d, M4B_TYPE_F32, R, 1, kHeads, 1) || d.nb[0] != 4 || d.nb[2] % 4 != 0 ||
        d.nb[2] < 4u * R || !d.data || !aligned(d.data, 4))
        return M4B_EINVAL;
    return M4B_OK;
}

// Partial records F32 [R + 4, 32, S] (contiguous, 16-byte aligned) of geometry g.
int check_partials(const m4b_tensor& p, int64_t max_splits, int g) {
    if (p.type != M4B_TYPE_F32 || p.ne[0] != kGeo[g].part || p.ne[1] != kHeads || p.ne[2] < 1 ||
        p.ne[3] != 1 || !packed3(p, 4) || !p.data || !aligned(p.data, 16))
        return M4B_EINVAL;
    if (max_splits > 0 && p.ne[2] > max_splits) return M4B_EINVAL;
    return M4B_OK;
}

// The geometry a record tensor belongs to (by its record width), or -1.
int record_geometry(const m4b_tensor& p) {
    if (p.ne[0] == kGeo[kGeomBaseline].part) return kGeomBaseline;
    if (p.ne[0] == kGeo[kGeomMistral].part) return kGeomMistral;
    return -1;
}

KqkvLaunch make_kqkv_launch(const m4b_kqkv_args& a, int g, int splits, float* part) {
    KqkvLaunch l;
    l.latent = kGeo[g].latent;
    l.q_token_stride = 0;
    l.kcache = a.src0.data;
    l.kcache_row_bytes = a.src0.nb[1];
    l.n_kv = a.src0.ne[1];
    l.q = static_cast<const float*>(a.src1.data);
    l.q_head_stride = static_cast<int64_t>(a.src1.nb[1] / 4);
    l.mask = static_cast<const float*>(a.src2.data);
    l.kq_scale = a.kq_scale;
    l.splits = splits;
    l.part = part;
    l.flags = a.flags;
    return l;
}

// Ragged batch (additive): kcache as for KQKV; q F32 [krow, 32, T]; seq_base / seq_len I32 [T];
// dst F32 [R, T, 32] (token stride nb[1], head stride nb[2]: ggml's kqv for T tokens).
int check_kqkv_ragged(const m4b_kqkv_ragged_args& a, int* geom) {
    m4b_kqkv_args k;
    std::memset(&k, 0, sizeof(k));
    k.src0 = a.kcache;
    k.kq_scale = a.kq_scale;
    const int64_t T = a.q.ne[2];
    if (T < 1 || T > kMaxSeqs) return M4B_EINVAL;
    k.src1 = a.q;
    k.src1.ne[2] = 1;   // the single-token check below covers dims 0..1
    int rc = check_kqkv_inputs(k, geom);
    if (rc != M4B_OK) return rc;
    if (a.q.ne[3] != 1 || a.q.nb[2] % 4 != 0) return M4B_EINVAL;
    if (a.kcache.ne[1] > (int64_t(1) << 30) - kTileKeys) return M4B_EINVAL;
    for (const m4b_tensor* t : {&a.seq_base, &a.seq_len})
        if (!type_ne(*t, M4B_TYPE_I32, T, 1, 1, 1) || t->nb[0] != 4 || !t->data ||
            !aligned(t->data, 4))
            return M4B_EINVAL;
    if (!f32_view(a.dst, kGeo[*geom].latent, T, kHeads)) return M4B_EINVAL;
    return M4B_OK;
}

uint64_t ragged_records(int64_t n_seq) { return static_cast<uint64_t>(kMaxSplits + n_seq - 1); }

// ---------------------------------------------------------------------------------------------
// PHASE
// ---------------------------------------------------------------------------------------------
// W_UV: F16 [512, 128, 32] or Q8_0 [256, 128, 32] (m4-phase.cu:212-213); sets the geometry.
int check_wuv(const m4b_tensor& w, int* geom) {
    if (type_ne(w, M4B_TYPE_Q8_0, 256, kVHead, kHeads, 1)) {
        if (!packed_q8(w) || !w.data || !aligned(w.data, 2)) return M4B_EINVAL;
        *geom = kGeomMistral;
        return M4B_OK;
    }
    if (!type_ne(w, M4B_TYPE_F16, kLatent, kVHead, kHeads, 1) || !packed3(w, 2) || !w.data ||
        !aligned(w.data, 16))
        return M4B_EINVAL;
    *geom = kGeomBaseline;
    return M4B_OK;
}

int check_phase_dst(const m4b_tensor& d) {
    if (!f32_view(d, kVHead, 1, kHeads) || d.nb[2] < 4u * kVHead) return M4B_EINVAL;
    return M4B_OK;
}

int check_attn(const m4b_tensor& x, int g) {   // F32 [R, 1, 32] with a head stride nb[2]
    const int R = kGeo[g].latent;
    if (!f32_view(x, R, 1, kHeads) || x.nb[2] < 4u * R) return M4B_EINVAL;
    return M4B_OK;
}

// PHASE selector 1 for T tokens: x F32 [R, T, 32], dst F32 [128, T, 32] (token stride nb[1],
// head stride nb[2]); T = 1 is the reference's op (ggml.c:3517-3539).
int check_wvb_tokens(const m4b_tensor& x, const m4b_tensor& d, int g) {
    const int64_t nt = x.ne[1];
    const int R = kGeo[g].latent;
    if (nt < 1 || nt > kMaxSeqs) return M4B_EINVAL;
    if (!f32_view(x, R, nt, kHeads) || x.nb[2] < 4u * R) return M4B_EINVAL;
    if (!f32_view(d, kVHead, nt, kHeads) || d.nb[2] < 4u * kVHead) return M4B_EINVAL;
    return M4B_OK;
}

// PHASE selector 0, the KV-write (m4-phase.cu:230-257): the Mistral-Small-4 geometry only.
//   src0 cur F32 [4096, 1]; src1 W_kva Q8_0 [4096, 320]; src2 kv_a_norm F32 [256];
//   src3 kcache F16 [320, N] (written in place); src4 kidx I64 [1]; src5 pos I32 [1];
//   dst Kcur F32 [320, 1]; op_params[8] (n_dims) == 64.
int check_kvwrite(const m4b_phase_args& a) {
    const m4b_tensor &cur = a.src[0], &w = a.src[1], &nw = a.src[2], &kc = a.src[3],
                     &kidx = a.src[4], &pos = a.src[5], &d = a.dst;
    if (!type_ne(cur, M4B_TYPE_F32, kKvwIn, 1, 1, 1) || cur.nb[0] != 4 || !cur.data ||
        !aligned(cur.data, 16))
        return M4B_EINVAL;
    if (!type_ne(w, M4B_TYPE_Q8_0, kKvwIn, 320, 1, 1) || w.nb[0] != kQ8Block ||
        w.nb[1] != static_cast<uint64_t>(kKvwIn / 32) * kQ8Block || !w.data || !aligned(w.data, 2))
        return M4B_EINVAL;
    // the tail moves value pairs: norm_w and Kcur 8-byte aligned, cache rows 4-byte aligned
    if (!type_ne(nw, M4B_TYPE_F32, 256, 1, 1, 1) || nw.nb[0] != 4 || !nw.data ||
        !aligned(nw.data, 8))
        return M4B_EINVAL;
    if (kc.type != M4B_TYPE_F16 || kc.ne[0] != 320 || kc.ne[1] < 1 || kc.ne[2] != 1 ||
        kc.ne[3] != 1 || kc.nb[0] != 2 || kc.nb[1] % 4 != 0 || kc.nb[1] < 640 || !kc.data ||
        !aligned(kc.data, 4))
        return M4B_EINVAL;
    if (!type_ne(kidx, M4B_TYPE_I64, 1, 1, 1, 1) || !kidx.data || !aligned(kidx.data, 8))
        return M4B_EINVAL;
    if (!type_ne(pos, M4B_TYPE_I32, 1, 1, 1, 1) || !pos.data || !aligned(pos.data, 4))
        return M4B_EINVAL;
    if (!type_ne(d, M4B_TYPE_F32, 320, 1, 1, 1) || d.nb[0] != 4 || !d.data || !aligned(d.data, 8))
        return M4B_EINVAL;
    if (a.op_params[8] != 64) return M4B_EINVAL;   // n_dims (m4-phase.cu:256)
    return M4B_OK;
}

// sets *geom for every selector (selector 0 is the Mistral geometry)
int check_phase(const m4b_phase_args& a, int* geom) {
    const int phase = a.op_params[0];
    switch (phase) {
        case 0: {
            // a BASELINE-shaped KV-write has no reference op (m4-phase.cu:230-257 is Mistral only)
            if (a.src[3].type == M4B_TYPE_F16 && a.src[3].ne[0] == kKRow) return M4B_ENOTSUP;
            *geom = kGeomMistral;
            return check_kvwrite(a);
        }
        case 1: {
            int rc = check_wuv(a.src[0], geom);
            if (rc != M4B_OK) return rc;
            return check_wvb_tokens(a.src[1], a.dst, *geom);
        }
        case 2: {
            int rc = check_wuv(a.src[0], geom);
            if (rc != M4B_OK) return rc;
            rc = check_partials(a.src[1], kMaxRecords, *geom);
            if (rc != M4B_OK) return rc;
            if (a.src[2].data != nullptr && check_attn(a.src[2], *geom) != M4B_OK) return M4B_EINVAL;
            return check_phase_dst(a.dst);
        }
        case 3: {   // merge records -> one record per head (additive, for the GPU exchange)
            const int g = record_geometry(a.src[1]);
            if (g < 0) return M4B_EINVAL;
            int rc = check_partials(a.src[1], kMaxRecords, g);
            if (rc != M4B_OK) return rc;
            const m4b_tensor& d = a.dst;
            if (d.type != M4B_TYPE_F32 || d.ne[0] != kGeo[g].part || d.ne[1] != kHeads ||
                d.ne[2] != 1 || d.ne[3] != 1 || !packed3(d, 4) || !d.data || !aligned(d.data, 16))
                return M4B_EINVAL;
            *geom = g;
            return M4B_OK;
        }
        default:   // m4-phase.cu:276 GGML_ABORT("unknown phase")
            return M4B_EINVAL;
    }
}

float param_f32(const int32_t* op_params, int i) {
    float f;
    std::memcpy(&f, op_params + i, sizeof(f));
    return f;
}

// YaRN correction dims, the host-side part of the rope (computed on the host by the reference's
// launcher too, m4-phase.cu:259-261): the rotary dims whose wavelength at the original context is
// between beta_fast and beta_slow rotations, corr(b) = n_dims ln(n_ctx_orig / (2 pi b)) /
// (2 ln base), clamped to [0, n_dims - 1] (the published YaRN rule as ggml applies it).
void yarn_corr_dims(int n_dims, int n_ctx_orig, float base, float beta_fast, float beta_slow,
                    float* lo, float* hi) {
    const float two_pi = 6.28318530717958647692f;
    const float a = n_dims * logf(n_ctx_orig / (beta_fast * two_pi)) / (2 * logf(base));
    const float b = n_dims * logf(n_ctx_orig / (beta_slow * two_pi)) / (2 * logf(base));
    *lo = std::max(0.0f, floorf(a));
    *hi = std::min(static_cast<float>(n_dims - 1), ceilf(b));
}

// PHASE selector 0 on a validated argument block (slab: see KvWriteLaunch).
int kvwrite(const m4b_phase_args& pa, int slab, int64_t slab_base, cudaStream_t s) {
    const m4b_phase_args* a = &pa;
    float* out = static_cast<float*>(a->dst.data);
    KvWriteLaunch k;
    k.cur = static_cast<const float*>(a->src[0].data);
    k.w = a->src[1].data;
    k.norm_w = static_cast<const float*>(a->src[2].data);
    k.kcache = a->src[3].data;
    k.kcache_row_stride = static_cast<int64_t>(a->src[3].nb[1] / 2);
    k.kcache_rows = a->src[3].ne[1];
    k.kidx = static_cast<const int64_t*>(a->src[4].data);
    k.pos = static_cast<const int32_t*>(a->src[5].data);
    k.kcur = out;
    // op_params (ggml.c:3464-3468, an int32 array): [1] freq_base [2] freq_scale
    // [3] ext_factor [4] attn_factor [5] beta_fast [6] beta_slow [7] eps [8] n_dims
    // [9] n_ctx_orig
    const float freq_base = param_f32(a->op_params, 1);
    k.freq_scale = param_f32(a->op_params, 2);
    k.ext_factor = param_f32(a->op_params, 3);
    k.attn_factor = param_f32(a->op_params, 4);
    const float beta_fast = param_f32(a->op_params, 5);
    const float beta_slow = param_f32(a->op_params, 6);
    k.eps = param_f32(a->op_params, 7);
    const int n_dims = a->op_params[8];
    yarn_corr_dims(n_dims, a->op_params[9], freq_base, beta_fast, beta_slow, &k.corr0, &k.corr1);
    k.theta_scale = powf(freq_base, -2.0f / static_cast<float>(n_dims));
    k.flags = a->flags;
    k.slab = slab;
    k.slab_base = slab_base;
    return status_of(launch_kvwrite(k, s));
}

}  // namespace
}  // namespace m4b

using namespace m4b;

extern "C" {

int m4b_abi_version(void) { return M4B_ABI_VERSION; }

const char* m4b_strerror(int code) {
    switch (code) {
        case M4B_OK: return "ok";
        case M4B_EINVAL: return "m4b: shape/type/stride/alignment contract violated";
        case M4B_ESCRATCH: return "m4b: scratch missing or too small";
        case M4B_ECUDA: return "m4b: CUDA runtime error";
        case M4B_EDEVICE: return "m4b: current device is not sm_100";
        case M4B_ENOTSUP: return "m4b: geometry or phase not implemented by this build";
        case M4B_ETIMEOUT: return "m4b: a kernel's bounded wait timed out";
        default: return "m4b: unknown status";
    }
}

int m4b_kqkv_max_splits(void) { return kMaxSplits; }

int m4b_kqkv_default_splits(int64_t n_kv) {
    if (n_kv < 1) return 0;
    int sms = kMaxSplits;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
            sms = v;
    } else {
        cudaGetLastError();
    }
    return default_splits(n_kv, sms);
}

uint64_t m4b_kqkv_scratch_bytes(int geometry, int64_t n_kv) {
    if (geometry < 0 || geometry > 1 || n_kv < 1) return 0;
    const int s = default_splits(n_kv, kMaxSplits);
    return static_cast<uint64_t>(s) * kHeads * kGeo[geometry].part * sizeof(float);
}

uint64_t m4b_phase_scratch_bytes(int phase) {
    return phase == 2 ? static_cast<uint64_t>(kHeads) * kLatent * sizeof(float) : 0;
}

int m4b_wkb(const m4b_wkb_args* a, m4b_stream_t stream) {
    if (!a) return M4B_EINVAL;
    int geom = 0;
    int rc = check_wkb(a->src0, a->src1, a->dst, &geom);
    if (rc != M4B_OK) return rc;
    if ((a->flags & M4B_FLAG_QCAT) &&   // the rope half sits after q_nope / after the latent
        (a->src1.nb[1] < 4u * (kGeo[geom].nope + 64) || a->dst.nb[1] < 4u * (kGeo[geom].latent + 64)))
        return M4B_EINVAL;
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    const Rows qr = {static_cast<int64_t>(a->src1.nb[1] / 4), static_cast<int64_t>(a->src1.nb[2] / 4)};
    const Rows outr = {static_cast<int64_t>(a->dst.nb[1] / 4), static_cast<int64_t>(a->dst.nb[2] / 4)};
    const int nt = static_cast<int>(a->src1.ne[2]);
    const float* q = static_cast<const float*>(a->src1.data);
    float* out = static_cast<float*>(a->dst.data);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (geom == kGeomMistral)
        return status_of(launch_wkb_q8(a->src0.data, q, qr, out, outr, nt, a->flags, s));
    return status_of(launch_wkb_f16(a->src0.data, q, qr, out, outr, nt, a->flags, s));
}

int m4b_kqkv(const m4b_kqkv_args* a, m4b_stream_t stream) {
    if (!a) return M4B_EINVAL;
    int geom = 0;
    int rc = check_kqkv(*a, &geom);
    if (rc != M4B_OK) return rc;
    int sms = 0;
    rc = device_check(&sms);
    if (rc != M4B_OK) return rc;
    const int64_t n_kv = a->src0.ne[1];
    const int splits = default_splits(n_kv, sms);
    const uint64_t need = static_cast<uint64_t>(splits) * kHeads * kGeo[geom].part * sizeof(float);
    if (!a->scratch || a->scratch_bytes < need || !aligned(a->scratch, 16)) return M4B_ESCRATCH;
    float* part = static_cast<float*>(a->scratch);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = launch_kqkv_partials(make_kqkv_launch(*a, geom, splits, part), s);
    if (e != cudaSuccess) return M4B_ECUDA;
    e = launch_kqkv_combine(part, splits, kGeo[geom].latent, static_cast<float*>(a->dst.data),
                            static_cast<int64_t>(a->dst.nb[2] / 4), a->flags & M4B_FLAG_PDL, s);
    return status_of(e);
}

int m4b_kqkv_partials(const m4b_kqkv_args* a, m4b_stream_t stream) {
    if (!a) return M4B_EINVAL;
    int geom = 0;
    int rc = check_kqkv_inputs(*a, &geom);
    if (rc != M4B_OK) return rc;
    rc = check_partials(a->dst, std::min<int64_t>(kMaxSplits, n_tiles(a->src0.ne[1])), geom);
    if (rc != M4B_OK) return rc;
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    const int splits = static_cast<int>(a->dst.ne[2]);
    return status_of(launch_kqkv_partials(
        make_kqkv_launch(*a, geom, splits, static_cast<float*>(a->dst.data)),
        reinterpret_cast<cudaStream_t>(stream)));
}

uint64_t m4b_kqkv_ragged_scratch_bytes(int64_t n_seq) {
    if (n_seq < 1 || n_seq > kMaxSeqs) return 0;
    return ragged_records(n_seq) * kHeads * kPartStride * sizeof(float);   // the wider geometry
}

int m4b_kqkv_ragged(const m4b_kqkv_ragged_args* a, m4b_stream_t stream) {
    if (!a) return M4B_EINVAL;
    int geom = 0;
    int rc = check_kqkv_ragged(*a, &geom);
    if (rc != M4B_OK) return rc;
    const int64_t T = a->q.ne[2];
    if (!a->scratch || a->scratch_bytes < m4b_kqkv_ragged_scratch_bytes(T) ||
        !aligned(a->scratch, 16))
        return M4B_ESCRATCH;
    int sms = 0;
    rc = device_check(&sms);
    if (rc != M4B_OK) return rc;
    const int G = std::min(sms, kMaxSplits);
    KqkvLaunch l;
    l.latent = kGeo[geom].latent;
    l.kcache = a->kcache.data;
    l.kcache_row_bytes = a->kcache.nb[1];
    l.n_kv = a->kcache.ne[1];
    l.q = static_cast<const float*>(a->q.data);
    l.q_head_stride = static_cast<int64_t>(a->q.nb[1] / 4);
    l.q_token_stride = static_cast<int64_t>(a->q.nb[2] / 4);
    l.mask = nullptr;
    l.kq_scale = a->kq_scale;
    l.splits = G;
    l.part = static_cast<float*>(a->scratch);
    l.flags = a->flags;
    l.seq_base = static_cast<const int32_t*>(a->seq_base.data);
    l.seq_len = static_cast<const int32_t*>(a->seq_len.data);
    l.n_seq = static_cast<int>(T);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = launch_kqkv_partials(l, s);
    if (e != cudaSuccess) return M4B_ECUDA;
    return status_of(launch_kqkv_ragged_combine(
        l.part, l.seq_base, l.seq_len, l.n_seq, l.n_kv, G, l.latent,
        static_cast<float*>(a->dst.data), static_cast<int64_t>(a->dst.nb[2] / 4),
        static_cast<int64_t>(a->dst.nb[1] / 4), a->flags & M4B_FLAG_PDL, s));
}

int m4b_phase(const m4b_phase_args* a, m4b_stream_t stream) {
    if (!a) return M4B_EINVAL;
    int geom = 0;
    int rc = check_phase(*a, &geom);
    if (rc != M4B_OK) return rc;
    const int phase = a->op_params[0];
    float* attn = nullptr;
    int64_t attn_hs = kGeo[geom].latent;
    if (phase == 2) {
        if (a->src[2].data != nullptr) {
            attn = static_cast<float*>(a->src[2].data);
            attn_hs = static_cast<int64_t>(a->src[2].nb[2] / 4);
        } else {
            if (!a->scratch || a->scratch_bytes < m4b_phase_scratch_bytes(2) ||
                !aligned(a->scratch, 16))
                return M4B_ESCRATCH;
            attn = static_cast<float*>(a->scratch);
        }
    }
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    float* out = static_cast<float*>(a->dst.data);
    const int64_t out_hs = static_cast<int64_t>(a->dst.nb[2] / 4);
    if (phase == 0) return kvwrite(*a, 0, 0, s);
    if (phase == 3) {
        return status_of(launch_kqkv_merge_records(static_cast<const float*>(a->src[1].data),
                                                   static_cast<int>(a->src[1].ne[2]),
                                                   kGeo[geom].latent, out, a->flags & M4B_FLAG_PDL,
                                                   s));
    }
    auto wvb = [&](const float* x, Rows xr, Rows outr, int nt, uint32_t flags) {
        if (geom == kGeomMistral) return launch_wvb_q8(a->src[0].data, x, xr, out, outr, nt, flags, s);
        return launch_wvb_f16(a->src[0].data, x, xr, out, outr, nt, flags, s);
    };
    if (phase == 1) {
        const Rows xr = {static_cast<int64_t>(a->src[1].nb[2] / 4),
                         static_cast<int64_t>(a->src[1].nb[1] / 4)};
        const Rows outr = {out_hs, static_cast<int64_t>(a->dst.nb[1] / 4)};
        return status_of(wvb(static_cast<const float*>(a->src[1].data), xr, outr,
                             static_cast<int>(a->src[1].ne[1]), a->flags));
    }
    // phase 2: merge the partial records, then W_UV -- one launch at the f16 geometry (attn is
    // written only when the caller passed src[2]), two at the Q8_0 geometry
    const int n_rec = static_cast<int>(a->src[1].ne[2]);
    if (geom != kGeomMistral && 2 * static_cast<size_t>(n_rec) * sizeof(float) <= 48 * 1024)
        return status_of(launch_kqkv_combine_wvb(
            static_cast<const float*>(a->src[1].data), n_rec, a->src[0].data,
            a->src[2].data != nullptr ? attn : nullptr, attn_hs, out, out_hs,
            a->flags & (M4B_FLAG_PDL | M4B_FLAG_EARLY_RELEASE), s));
    cudaError_t e = launch_kqkv_combine(static_cast<const float*>(a->src[1].data),
                                        static_cast<int>(a->src[1].ne[2]), kGeo[geom].latent, attn,
                                        attn_hs, a->flags & M4B_FLAG_PDL, s);
    if (e != cudaSuccess) return M4B_ECUDA;
    return status_of(wvb(attn, Rows{attn_hs, 0}, Rows{out_hs, 0}, 1, a->flags & M4B_FLAG_PDL));
}

int m4b_phase_kvwrite_slab(const m4b_phase_args* a, int64_t slab_base, m4b_stream_t stream) {
    if (!a || a->op_params[0] != 0 || slab_base < 0) return M4B_EINVAL;
    int geom = 0;
    int rc = check_phase(*a, &geom);
    if (rc != M4B_OK) return rc;
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    return kvwrite(*a, 1, slab_base, reinterpret_cast<cudaStream_t>(stream));
}

int m4b_supports_op(int op, const m4b_tensor* srcs, int n_srcs, const m4b_tensor* dst,
                    const int32_t* op_params) {
    if (!srcs || !dst) return 0;
    int geom = 0;
    switch (op) {
        case 0: {
            if (n_srcs < 2) return 0;
            return check_wkb(srcs[0], srcs[1], *dst, &geom) == M4B_OK;
        }
        case 1: {
            if (n_srcs < 2) return 0;
            if (n_srcs >= 5 && srcs[3].data != nullptr) {   // the ragged batch form
                if (n_srcs > 2 && srcs[2].data != nullptr) return 0;   // windows, not a mask
                m4b_kqkv_ragged_args r;
                std::memset(&r, 0, sizeof(r));
                r.kcache = srcs[0];
                r.q = srcs[1];
                r.seq_base = srcs[3];
                r.seq_len = srcs[4];
                r.dst = *dst;
                r.kq_scale = op_params ? *reinterpret_cast<const float*>(op_params) : 1.0f;
                return check_kqkv_ragged(r, &geom) == M4B_OK;
            }
            m4b_kqkv_args a;
            std::memset(&a, 0, sizeof(a));
            a.src0 = srcs[0];
            a.src1 = srcs[1];
            if (n_srcs >= 3) a.src2 = srcs[2];
            a.dst = *dst;
            a.kq_scale = op_params ? *reinterpret_cast<const float*>(op_params) : 1.0f;
            return check_kqkv(a, &geom) == M4B_OK;
        }
        case 2: {
            if (!op_params) return 0;
            m4b_phase_args a;
            std::memset(&a, 0, sizeof(a));
            for (int i = 0; i < n_srcs && i < 6; ++i) a.src[i] = srcs[i];
            a.dst = *dst;
            std::memcpy(a.op_params, op_params, sizeof(int32_t) * 10);
            return check_phase(a, &geom) == M4B_OK;
        }
        default:
            return 0;
    }
}

int m4b_resolve_flag(int flag, int gpu_core, int nt, int ragged_ok, int* enabled) {
    if (!enabled) return M4B_EINVAL;
    *enabled = 0;
    if (flag < -1 || flag > 1) return M4B_EINVAL;
    if (flag == 1 && !gpu_core) return M4B_EINVAL;                  // m1_engine.cpp:2182-2197
    if (flag == 1 && nt > 1 && !ragged_ok) return M4B_EINVAL;       // m1_engine.cpp:2100-2110
    const int on = (flag < 0) ? (gpu_core != 0) : (flag == 1);
    *enabled = on && (nt == 1 || ragged_ok);                        // m1_layer.cpp:283-297
    return M4B_OK;
}

int m4b_last_cuda_error(const char** name) {
    const int e = last_cuda_error().exchange(0);
    if (name) *name = cudaGetErrorName(static_cast<cudaError_t>(e));
    return e;
}

int m4b_set_wait_limit_cycles(int64_t cycles) {
    const long long v = cycles > 0 ? static_cast<long long>(cycles) : M4B_WAIT_LIMIT_CYCLES;
    if (note(cudaMemcpyToSymbol(g_wait_limit, &v, sizeof(v))) != cudaSuccess) return M4B_ECUDA;
    return note(cudaDeviceSynchronize()) == cudaSuccess ? M4B_OK : M4B_ECUDA;
}

int m4b_device_status(m4b_stream_t stream) {
    unsigned int v = 0;
    if (cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
        return M4B_ECUDA;
    if (cudaMemcpyFromSymbol(&v, g_status, sizeof(v)) != cudaSuccess) return M4B_ECUDA;
    if (v != 0) {
        const unsigned int zero = 0;
        if (cudaMemcpyToSymbol(g_status, &zero, sizeof(zero)) != cudaSuccess) return M4B_ECUDA;
        return v == DEV_STATUS_BADSEQ ? M4B_EINVAL : M4B_ETIMEOUT;
    }
    return M4B_OK;
}

}  // extern "C"
