// m4b_q8.cu -- the Mistral-Small-4 geometry's Q8_0 kernels (engine/m1_layer.h:47-55):
//   GGML_OP_M4_WKB    q_abs[t][h][r] = W_UK[h][r] . Q8(q_nope[t][h])      Q8_0 [64, 256, 32]
//   M4_PHASE 1 (WVB)  out[t][h][j]   = W_UV[h][j] . Q8(x[t][h])           Q8_0 [256, 128, 32]
//   M4_PHASE 0        the KV-write: Kcur = W_kva . Q8(cur) (Q8_0 [4096, 320]), RMS norm of the
//                     latent part times its weight, YaRN rope of the rope part, the f16 row
//                     scattered into the cache at a row read on the device.
//
// Numerics follow the reference's fused kernels, which replicate ggml-cuda's MMVQ path rather
// than an exact f32 dot (m4-wkb.cu:14-25, m4-phase.cu:35-40): the f32 activation is quantized per
// 32-value block to int8 with scale d = amax/127 (the dot uses f16(d)), the block dot is an int32
// sum of int8 products, and blocks combine as (d_w * f16(d_x)) * sum in the reference's order:
//   WKB   q = roundf(x / d), blocks summed in order                       (m4-wkb.cu:36-52)
//   WVB   q = roundf(x * (1/d)); lane l of a warp owns element l of every block, then a
//         butterfly sum over the lanes                                     (m4-phase.cu:62-88)
//   KV-write gemv: thread b owns block b of a row, warp butterflies, then the 4 warp partials
//         summed in order                                                  (m4-phase.cu:97-125)
// Each is a small HBM / latency-bound gemv (0.5-1.4 MB of weights): CUDA cores with dp4a, no
// tensor cores.
#include <cuda_fp16.h>

#include "m4b_internal.h"
#include "m4b_ptx.cuh"

namespace m4b {
namespace q8 {

constexpr int QK = 32;          // values per Q8_0 block
constexpr int BLK_BYTES = 34;   // f16 scale + 32 int8

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

__device__ __forceinline__ float warp_amax(float v) {
    v = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half(x)); }

// ---- WKB.  8192 rows of 64 values (2 blocks, 68 B: 4-byte aligned).  CTA = (head, 64 rows),
// one row per thread held in registers as 17 words; the head's activation blocks are quantized
// once per CTA into shared memory, for every token of the batch.
constexpr int WKB_ROWS = 64;
constexpr int WKB_NOPE = 64;
constexpr int WKB_R = 256;

__global__ void __launch_bounds__(WKB_ROWS)
wkb_q8_kernel(const uint8_t* __restrict__ w, const float* __restrict__ q, Rows qr,
              float* __restrict__ out, Rows outr, int nt, int qcat) {
    __shared__ __align__(16) int8_t s_xq[kMaxSeqs][2][QK];
    __shared__ float s_xd[kMaxSeqs][2];
    const int h = blockIdx.x;
    const int r = blockIdx.y * WKB_ROWS + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t* wr = reinterpret_cast<const uint32_t*>(w + static_cast<size_t>(h * WKB_R + r) * 68);
    uint32_t wv[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) wv[i] = __ldg(wr + i);
    pdl_wait();
    if (qcat) wkb_concat_rope(q, qr, 2 * QK, out, outr, WKB_R, nt, h, blockIdx.y, gridDim.y, WKB_ROWS);
    // quantize (token, block) pairs: warp-wide amax, lane = element
    for (int pb = warp; pb < 2 * nt; pb += WKB_ROWS / 32) {
        const int t = pb >> 1, b = pb & 1;
        const float x = q[t * qr.ts + h * qr.hs + b * QK + lane];
        const float amax = warp_amax(x);
        const float d = amax / 127.0f;
        s_xq[t][b][lane] = static_cast<int8_t>(amax == 0.0f ? 0 : static_cast<int>(roundf(x / d)));
        if (lane == 0) s_xd[t][b] = f16_round(d);
    }
    __syncthreads();
    // block 0's quants start at byte 2 (straddle words), block 1's at byte 36 = word 9
    uint32_t w0[8], w1[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        w0[k] = __funnelshift_r(wv[k], wv[k + 1], 16);
        w1[k] = wv[9 + k];
    }
    const float wd0 = __half2float(__ushort_as_half(static_cast<unsigned short>(wv[0] & 0xffffu)));
    const float wd1 = __half2float(__ushort_as_half(static_cast<unsigned short>(wv[8] >> 16)));
    for (int t = 0; t < nt; ++t) {
        const int* x0 = reinterpret_cast<const int*>(s_xq[t][0]);
        const int* x1 = reinterpret_cast<const int*>(s_xq[t][1]);
        int s0 = 0, s1 = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            s0 = __dp4a(static_cast<int>(w0[k]), x0[k], s0);
            s1 = __dp4a(static_cast<int>(w1[k]), x1[k], s1);
        }
        float acc = 0.0f;
        acc += wd0 * s_xd[t][0] * static_cast<float>(s0);
        acc += wd1 * s_xd[t][1] * static_cast<float>(s1);
        out[t * outr.ts + h * outr.hs + r] = acc;
    }
}

// ---- WVB.  4096 rows of 256 values (8 blocks, 272 B).  CTA = (head, 8 rows), warp = row,
// lane = element of every block (coalesced byte loads across the warp, as 2-byte-aligned Q8_0
// blocks allow).  The head's 8 activation blocks are quantized once per CTA per token.
constexpr int WVB_R = 256;
constexpr int WVB_V = 128;
constexpr int WVB_NB = WVB_R / QK;   // 8

__global__ void __launch_bounds__(256)
wvb_q8_kernel(const uint8_t* __restrict__ w, const float* __restrict__ x, Rows xr,
              float* __restrict__ out, Rows outr, int nt) {
    __shared__ int8_t s_xq[kMaxSeqs][WVB_NB][QK];
    __shared__ float s_xd[kMaxSeqs][WVB_NB];
    const int h = blockIdx.x >> 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = (blockIdx.x & 15) * 8 + warp;
    const uint8_t* wr = w + static_cast<size_t>(h * WVB_V + j) * (WVB_NB * BLK_BYTES);
    float wd[WVB_NB];
    int wq[WVB_NB];
#pragma unroll
    for (int b = 0; b < WVB_NB; ++b) {
        wd[b] = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(
            wr + b * BLK_BYTES))));
        wq[b] = static_cast<int8_t>(__ldg(wr + b * BLK_BYTES + 2 + lane));
    }
    pdl_wait();
    for (int pb = warp; pb < WVB_NB * nt; pb += 8) {
        const int t = pb / WVB_NB, b = pb % WVB_NB;
        const float v = x[t * xr.ts + h * xr.hs + b * QK + lane];
        const float amax = warp_amax(v);
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        s_xq[t][b][lane] = static_cast<int8_t>(static_cast<int>(roundf(v * id)));
        if (lane == 0) s_xd[t][b] = f16_round(d);
    }
    __syncthreads();
    for (int t = 0; t < nt; ++t) {
        float acc = 0.0f;
#pragma unroll
        for (int b = 0; b < WVB_NB; ++b)
            acc += wd[b] * s_xd[t][b] * static_cast<float>(wq[b] * static_cast<int>(s_xq[t][b][lane]));
        acc = warp_sum(acc);
        if (lane == 0) out[t * outr.ts + h * outr.hs + j] = acc;
    }
}

// ---- KV-write.  gemv: grid = 320 output rows, block = 128 threads, thread b owns block b of the
// row and the 32 input values it multiplies (quantized by that thread: no cross-thread
// dependency).  The 320 pre-norm outputs go to dst (Kcur), which the tail then finishes in place.
constexpr int KVW_IN = 4096;
constexpr int KVW_NB = KVW_IN / QK;   // 128
constexpr int KVW_LAT = 256;
constexpr int KVW_ROPE = 64;
constexpr int KVW_ROW = KVW_LAT + KVW_ROPE;   // 320

__global__ void __launch_bounds__(KVW_NB)
kvwrite_gemv_kernel(const float* __restrict__ cur, const uint8_t* __restrict__ w,
                    float* __restrict__ kcur) {
    __shared__ float s_part[KVW_NB / 32];
    const int o = blockIdx.x;
    const int tid = threadIdx.x;
    const uint8_t* wb = w + static_cast<size_t>(o) * (KVW_NB * BLK_BYTES) + tid * BLK_BYTES;
    const float wd = __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(wb))));
    int wq[QK / 4];
#pragma unroll
    for (int k = 0; k < QK / 4; ++k) {   // bytes 2..33: 2-byte aligned, assemble words
        const unsigned short lo = __ldg(reinterpret_cast<const unsigned short*>(wb + 2 + 4 * k));
        const unsigned short hi = __ldg(reinterpret_cast<const unsigned short*>(wb + 4 + 4 * k));
        wq[k] = static_cast<int>(static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16));
    }
    pdl_wait();
    const float4* xb = reinterpret_cast<const float4*>(cur + tid * QK);
    float xv[QK];
#pragma unroll
    for (int k = 0; k < QK / 4; ++k) {
        const float4 v = xb[k];
        xv[4 * k] = v.x; xv[4 * k + 1] = v.y; xv[4 * k + 2] = v.z; xv[4 * k + 3] = v.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < QK; ++k) amax = fmaxf(amax, fabsf(xv[k]));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    int sum = 0;
#pragma unroll
    for (int k = 0; k < QK / 4; ++k) {
        uint32_t packed = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            packed |= (static_cast<uint32_t>(static_cast<int>(roundf(xv[4 * k + i] * id))) & 0xffu)
                      << (8 * i);
        sum = __dp4a(wq[k], static_cast<int>(packed), sum);
    }
    float acc = wd * f16_round(d) * static_cast<float>(sum);
    acc = warp_sum(acc);
    if ((tid & 31) == 0) s_part[tid >> 5] = acc;
    __syncthreads();
    if (tid == 0) kcur[o] = s_part[0] + s_part[1] + s_part[2] + s_part[3];
}

// ---- KV-write tail: finishes the 320 pre-norm values the gemv left in Kcur.
//   Kcur[0, 256)   = kv[0, 256) / sqrt(mean(kv[0, 256)^2) + eps) * norm_w      (ggml rms_norm, mul)
//   Kcur[256, 320) = the 32 pairs (kv[256 + 2p], kv[257 + 2p]) rotated by the YaRN angle of pair p
//                    at position pos (ggml rope, NORMAL mode, ggml-cpu/ops.cpp:6179-6201)
// then f16(Kcur) into cache row kidx[0].  One CTA of 5 warps; thread t owns the value pair
// (2t, 2t + 1): warps 0-3 the 128 latent pairs, warp 4 the 32 rope pairs, so every load and store
// moves a float2 (a half2 into the cache).  The sum of squares is reduced per warp by shuffles;
// each thread then adds the 4 warp totals itself, in warp order, so the scale needs no second
// barrier.  kidx and pos are read on the device; a cache row outside [0, n_rows) is not written
// and sets the device status.
struct RopeArgs {
    float eps, freq_scale, ext_factor, attn_factor, theta_scale, corr0, corr1;
};

constexpr int KVT_LAT_PAIRS = KVW_LAT / 2;           // 128: warps 0-3
constexpr int KVT_ROPE_PAIRS = KVW_ROPE / 2;         // 32: warp 4
constexpr int KVT_THREADS = KVT_LAT_PAIRS + KVT_ROPE_PAIRS;

// ggml's YaRN blend for pair p: 1 below corr0, 0 above corr1, linear between
// (rope_yarn_ramp, evaluated at i0 / 2 = p).
__device__ __forceinline__ float yarn_ramp(float corr_lo, float corr_hi, int p) {
    const float t = (static_cast<float>(p) - corr_lo) / fmaxf(0.001f, corr_hi - corr_lo);
    return 1.0f - fminf(1.0f, fmaxf(0.0f, t));
}

// The rotation (cos, sin), magnitude included, of pair p at position pos (ggml rope_yarn).
__device__ __forceinline__ float2 yarn_rotation(const RopeArgs& ra, int pos, int p) {
    const float ang_extrap = static_cast<float>(pos) * powf(ra.theta_scale, static_cast<float>(p));
    const float ang_interp = ra.freq_scale * ang_extrap;
    float ang = ang_interp, mag = ra.attn_factor;
    if (ra.ext_factor != 0.0f) {
        const float blend = yarn_ramp(ra.corr0, ra.corr1, p) * ra.ext_factor;
        ang = ang_interp * (1.0f - blend) + ang_extrap * blend;
        mag *= 1.0f + 0.1f * logf(1.0f / ra.freq_scale);
    }
    return make_float2(cosf(ang) * mag, sinf(ang) * mag);
}

__global__ void __launch_bounds__(KVT_THREADS)
kvwrite_tail_kernel(float* __restrict__ kcur, const float* __restrict__ nw,
                    __half* __restrict__ kcache, int64_t row_stride, int64_t n_rows,
                    const int64_t* __restrict__ kidx, const int32_t* __restrict__ posv,
                    RopeArgs ra, int slab, int64_t slab_base) {
    __shared__ float s_sumsq[KVT_LAT_PAIRS / 32];
    const int t = threadIdx.x;
    const int wp = t >> 5;
    pdl_wait();
    const int64_t cache_row = kidx[0];
    const int64_t local_row = slab ? cache_row - slab_base : cache_row;
    float2* kc2 = reinterpret_cast<float2*>(kcur);
    const float2 pr = kc2[t];                 // this thread's pair of pre-norm values
    float sumsq = t < KVT_LAT_PAIRS ? pr.x * pr.x + pr.y * pr.y : 0.0f;
    sumsq = warp_sum(sumsq);
    if (wp < KVT_LAT_PAIRS / 32 && (t & 31) == 0) s_sumsq[wp] = sumsq;
    float2 res;
    if (t < KVT_LAT_PAIRS) {
        const float2 g = reinterpret_cast<const float2*>(nw)[t];
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < KVT_LAT_PAIRS / 32; ++w) tot += s_sumsq[w];
        const float inv_rms = rsqrtf(tot / static_cast<float>(KVW_LAT) + ra.eps);
        res = make_float2(pr.x * inv_rms * g.x, pr.y * inv_rms * g.y);
    } else {
        const float2 cs = yarn_rotation(ra, posv[0], t - KVT_LAT_PAIRS);
        __syncthreads();
        res = make_float2(pr.x * cs.x - pr.y * cs.y, pr.x * cs.y + pr.y * cs.x);
    }
    kc2[t] = res;                             // each thread rewrites only the pair it read
    if (local_row >= 0 && local_row < n_rows) {
        reinterpret_cast<__half2*>(kcache + local_row * row_stride)[t] = __float22half2_rn(res);
    } else if (t == 0 && (!slab || cache_row < 0)) {
        // one cache: a row outside it is an error; a slab: only a negative row is, any other row
        // belongs to another GPU's slab
        atomicExch(&g_status, DEV_STATUS_BADSEQ);
    }
}

}  // namespace q8

cudaError_t launch_wkb_q8(const void* w, const float* q, Rows qr, float* out, Rows outr, int nt,
                          uint32_t flags, cudaStream_t stream) {
    using namespace q8;
    return launch(wkb_q8_kernel, dim3(kHeads, WKB_R / WKB_ROWS), dim3(WKB_ROWS), 0, stream, flags,
                  static_cast<const uint8_t*>(w), q, qr, out, outr, nt,
                  (flags & M4B_FLAG_QCAT) ? 1 : 0);
}

cudaError_t launch_wvb_q8(const void* w, const float* x, Rows xr, float* out, Rows outr, int nt,
                          uint32_t flags, cudaStream_t stream) {
    using namespace q8;
    return launch(wvb_q8_kernel, dim3(kHeads * (WVB_V / 8)), dim3(256), 0, stream, flags,
                  static_cast<const uint8_t*>(w), x, xr, out, outr, nt);
}

cudaError_t launch_kvwrite(const KvWriteLaunch& a, cudaStream_t stream) {
    using namespace q8;
    cudaError_t e = launch(kvwrite_gemv_kernel, dim3(KVW_ROW), dim3(KVW_NB), 0, stream, a.flags,
                           a.cur, static_cast<const uint8_t*>(a.w), a.kcur);
    if (e != cudaSuccess) return e;
    RopeArgs ra = {a.eps, a.freq_scale, a.ext_factor, a.attn_factor, a.theta_scale, a.corr0, a.corr1};
    return launch(kvwrite_tail_kernel, dim3(1), dim3(KVT_THREADS), 0, stream, a.flags | M4B_FLAG_PDL,
                  a.kcur, a.norm_w, static_cast<__half*>(a.kcache), a.kcache_row_stride,
                  a.kcache_rows, a.kidx, a.pos, ra, a.slab, a.slab_base);
}

}  // namespace m4b
