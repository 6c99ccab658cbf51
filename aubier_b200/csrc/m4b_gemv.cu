// m4b_gemv.cu -- the two per-head absorption gemvs of the MLA decode path on sm_100a:
//   GGML_OP_M4_WKB     q_abs[h][r] = sum_k W_UK[h][r][k] * f16(q_nope[h][k])   (32 x 512 x 128)
//   M4_PHASE WVB (1)   out[h][j]   = sum_r W_UV[h][j][r] * f16(x[h][r])        (32 x 128 x 512)
// Both are 4 MiB of f16 weights read once against a 16 KB / 64 KB activation: HBM-bound streams,
// not GEMMs (each weight element is used exactly once), so they run on CUDA cores with 16-byte
// vector loads, several rows in flight per warp and a shuffle reduction -- no tensor cores.
// Both take a batch of nt tokens (the ragged decode path); the reference's ops are nt = 1.
// The activation is rounded to f16 (round to nearest even) before the dot, as the reference CPU
// graph's F16 mul_mat does with its F32 src1 (ggml-cpu.c:1330-1375); products accumulate in f32.
// Reference kernels replaced: m4-wkb.cu:55-69 (Q8_0 geometry) and m4-phase.cu:52-89.
//
// PDL: the weight rows do not depend on the preceding kernel, so they are loaded into registers
// BEFORE griddepcontrol.wait; only the activation read waits.  WKB alone releases its dependent
// (the KQKV launch) as soon as its weights are in flight: KQKV's CTAs then set up and, with a
// static cache, start streaming it on the SMs WKB leaves free, while WKB finishes (measured
// ~0.6 us per layer-step on the 36-layer chain).  Releasing early from every kernel was measured
// ~7% slower: the next layer's KQKV grid then held the SMs while this layer's small kernels
// still had to run.
#include <cuda_fp16.h>

#include "m4b_internal.h"
#include "m4b_ptx.cuh"

namespace m4b {
namespace gemv {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float round_f16(float x) { return __half2float(__float2half_rn(x)); }

// ---- WKB: 16384 rows of 128 f16 (256 B).  A half-warp covers one row (16 lanes x 16 B); a warp
// handles 8 consecutive rows of one head (4 loads in flight per lane); 8 warps per CTA.  A batch
// of nt tokens reuses the rows held in registers: the weights are read from HBM once.
constexpr int WKB_ROWS_PER_WARP = 8;
constexpr int WKB_THREADS = 256;

__global__ void __launch_bounds__(WKB_THREADS)
wkb_f16_kernel(const __half* __restrict__ w, const float* __restrict__ q, Rows qr,
               float* __restrict__ out, Rows outr, int nt, int qcat) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * (WKB_THREADS / 32) + warp) * WKB_ROWS_PER_WARP;
    const int h = row0 / kLatent;
    const int r0 = row0 % kLatent;
    const int hw = lane >> 4;        // which of the warp's two rows per load
    const int l16 = lane & 15;       // k = 8*l16 .. 8*l16+7

    uint4 wv[WKB_ROWS_PER_WARP / 2];
#pragma unroll
    for (int it = 0; it < WKB_ROWS_PER_WARP / 2; ++it) {
        const int row = row0 + 2 * it + hw;
        wv[it] = ldg_stream(w + static_cast<size_t>(row) * kNope + 8 * l16);
    }
    pdl_launch_dependents();
    pdl_wait();
    if (qcat) {   // the kLatent / 64 CTAs of head h share its tokens
        constexpr int per_head = kLatent / (WKB_ROWS_PER_WARP * (WKB_THREADS / 32));
        wkb_concat_rope(q, qr, kNope, out, outr, kLatent, nt, h, blockIdx.x % per_head, per_head,
                        WKB_THREADS);
    }
    for (int t = 0; t < nt; ++t) {
        const float* qt = q + t * qr.ts + h * qr.hs + 8 * l16;
        float qf[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) qf[j] = round_f16(qt[j]);
        float* ot = out + t * outr.ts + h * outr.hs + r0;
#pragma unroll
        for (int it = 0; it < WKB_ROWS_PER_WARP / 2; ++it) {
            float wf[8];
            unpack8(wv[it], wf);
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fmaf(wf[j], qf[j], acc);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (l16 == 0) ot[2 * it + hw] = acc;
        }
    }
}

// ---- WVB: 4096 rows of 512 f16 (1 KB).  A warp covers a row with two 16-B loads per lane and
// handles 2 rows (4 loads in flight per lane); 8 warps per CTA, 256 CTAs.  Tokens as for WKB.
constexpr int WVB_ROWS_PER_WARP = 2;
constexpr int WVB_THREADS = 256;

__global__ void __launch_bounds__(WVB_THREADS)
wvb_f16_kernel(const __half* __restrict__ w, const float* __restrict__ x, Rows xr,
               float* __restrict__ out, Rows outr, int nt) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * (WVB_THREADS / 32) + warp) * WVB_ROWS_PER_WARP;
    const int h = row0 / kVHead;
    const int j0 = row0 % kVHead;

    uint4 wv[WVB_ROWS_PER_WARP][2];
#pragma unroll
    for (int it = 0; it < WVB_ROWS_PER_WARP; ++it)
#pragma unroll
        for (int u = 0; u < 2; ++u)
            wv[it][u] = ldg_stream(w + static_cast<size_t>(row0 + it) * kLatent + 256 * u + 8 * lane);
    pdl_wait();
    for (int t = 0; t < nt; ++t) {
        const float* xt = x + t * xr.ts + h * xr.hs;
        float xf[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float4* xp = reinterpret_cast<const float4*>(xt + 256 * u + 8 * lane);
            if ((reinterpret_cast<uintptr_t>(xp) & 15) == 0) {
                const float4 a = xp[0], b = xp[1];
                xf[u][0] = a.x; xf[u][1] = a.y; xf[u][2] = a.z; xf[u][3] = a.w;
                xf[u][4] = b.x; xf[u][5] = b.y; xf[u][6] = b.z; xf[u][7] = b.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) xf[u][j] = xt[256 * u + 8 * lane + j];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) xf[u][j] = round_f16(xf[u][j]);
        }
#pragma unroll
        for (int it = 0; it < WVB_ROWS_PER_WARP; ++it) {
            float acc = 0.0f;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                float wf[8];
                unpack8(wv[it][u], wf);
#pragma unroll
                for (int j = 0; j < 8; ++j) acc = fmaf(wf[j], xf[u][j], acc);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
            if (lane == 0) out[t * outr.ts + h * outr.hs + j0 + it] = acc;
        }
    }
}

// ---- Token batches (nt > 1, the ragged decode path).  The loops above would read each token's
// activation from L2 inside the token loop -- one dependent L2 round trip per token -- and reduce
// every (row, token) dot with its own shuffle tree.  Here a CTA (one head: 64 WKB rows or 16 WVB
// rows) first stages all nt activations of its head in shared memory, rounded to f16 (one L2 round
// trip), and a chunk of tokens is reduced at once: each lane holds rows x tokens partial dots and
// one xor butterfly leaves every lane with one finished (row, token) sum.  The per-lane dot and the
// butterfly's pairing are those of the single-token kernels, so results are bit-identical to them.

// Sum each of N values over the N lanes of an xor group (lanes differing in their low log2(N)
// bits); afterwards lane L holds the sum of value index (L & (N - 1)).
template <int N>
__device__ __forceinline__ float xor_transpose_reduce(float (&v)[N], int lane) {
#pragma unroll
    for (int n = N, off = N / 2; n > 1; n >>= 1, off >>= 1) {
        const bool upper = (lane & off) != 0;
        const int half = n >> 1;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    return v[0];
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Stage n_units units of 8 activations (f32 -> f16, round to nearest even) of one head:
// unit i = token i / upt, columns 8 * (i % upt) .. +7; tokens >= nt are zero.
__device__ __forceinline__ void stage_tokens(__half* xs, const float* __restrict__ x, Rows xr, int h,
                                             int nt, int ntp, int upt, int nthreads) {
    for (int i = threadIdx.x; i < ntp * upt; i += nthreads) {
        const int t = i / upt, u = i % upt;
        uint4 pk = make_uint4(0u, 0u, 0u, 0u);
        if (t < nt) {
            const float* src = x + static_cast<size_t>(t) * xr.ts + static_cast<size_t>(h) * xr.hs + 8 * u;
            float f[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = src[j];
            pk.x = pack_h2(f[0], f[1]);
            pk.y = pack_h2(f[2], f[3]);
            pk.z = pack_h2(f[4], f[5]);
            pk.w = pack_h2(f[6], f[7]);
        }
        reinterpret_cast<uint4*>(xs)[i] = pk;
    }
}

constexpr int WKB_TCH = 4;    // tokens per butterfly: 4 row pairs x 4 tokens = 16 values, 16 lanes
constexpr int WVB_TCH = 16;   // 2 rows x 16 tokens = 32 values, 32 lanes

__global__ void __launch_bounds__(WKB_THREADS)
wkb_f16_batch_kernel(const __half* __restrict__ w, const float* __restrict__ q, Rows qr,
                     float* __restrict__ out, Rows outr, int nt, int qcat) {
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    __half* xs = reinterpret_cast<__half*>(dyn_smem);   // [ntp][kNope]
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * (WKB_THREADS / 32) + warp) * WKB_ROWS_PER_WARP;
    const int h = (blockIdx.x * (WKB_THREADS / 32) * WKB_ROWS_PER_WARP) / kLatent;   // one head per CTA
    const int r0 = row0 % kLatent;
    const int hw = lane >> 4;
    const int l16 = lane & 15;
    const int ntp = (nt + WKB_TCH - 1) / WKB_TCH * WKB_TCH;

    uint4 wv[WKB_ROWS_PER_WARP / 2];
#pragma unroll
    for (int it = 0; it < WKB_ROWS_PER_WARP / 2; ++it)
        wv[it] = ldg_stream(w + static_cast<size_t>(row0 + 2 * it + hw) * kNope + 8 * l16);
    pdl_launch_dependents();
    pdl_wait();
    if (qcat) {   // the kLatent / 64 CTAs of head h share its tokens
        constexpr int per_head = kLatent / (WKB_ROWS_PER_WARP * (WKB_THREADS / 32));
        wkb_concat_rope(q, qr, kNope, out, outr, kLatent, nt, h, blockIdx.x % per_head, per_head,
                        WKB_THREADS);
    }
    stage_tokens(xs, q, qr, h, nt, ntp, kNope / 8, WKB_THREADS);
    float wf[WKB_ROWS_PER_WARP / 2][8];
#pragma unroll
    for (int it = 0; it < WKB_ROWS_PER_WARP / 2; ++it) unpack8(wv[it], wf[it]);
    __syncthreads();
    for (int c = 0; c < ntp; c += WKB_TCH) {
        float v[16];
#pragma unroll
        for (int tt = 0; tt < WKB_TCH; ++tt) {
            float xf[8];
            unpack8(*reinterpret_cast<const uint4*>(xs + (c + tt) * kNope + 8 * l16), xf);
#pragma unroll
            for (int it = 0; it < WKB_ROWS_PER_WARP / 2; ++it) {
                float acc = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; ++j) acc = fmaf(wf[it][j], xf[j], acc);
                v[WKB_TCH * it + tt] = acc;
            }
        }
        const float r = xor_transpose_reduce<16>(v, lane);
        const int it = l16 / WKB_TCH, t = c + l16 % WKB_TCH;
        if (t < nt) out[static_cast<size_t>(t) * outr.ts + h * outr.hs + r0 + 2 * it + hw] = r;
    }
}

__global__ void __launch_bounds__(WVB_THREADS)
wvb_f16_batch_kernel(const __half* __restrict__ w, const float* __restrict__ x, Rows xr,
                     float* __restrict__ out, Rows outr, int nt) {
    extern __shared__ __align__(16) uint8_t dyn_smem[];
    __half* xs = reinterpret_cast<__half*>(dyn_smem);   // [ntp][kLatent]
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * (WVB_THREADS / 32) + warp) * WVB_ROWS_PER_WARP;
    const int h = (blockIdx.x * (WVB_THREADS / 32) * WVB_ROWS_PER_WARP) / kVHead;   // one head per CTA
    const int j0 = row0 % kVHead;
    const int ntp = (nt + WVB_TCH - 1) / WVB_TCH * WVB_TCH;

    uint4 wv[WVB_ROWS_PER_WARP][2];
#pragma unroll
    for (int it = 0; it < WVB_ROWS_PER_WARP; ++it)
#pragma unroll
        for (int u = 0; u < 2; ++u)
            wv[it][u] = ldg_stream(w + static_cast<size_t>(row0 + it) * kLatent + 256 * u + 8 * lane);
    pdl_wait();
    stage_tokens(xs, x, xr, h, nt, ntp, kLatent / 8, WVB_THREADS);
    float wf[WVB_ROWS_PER_WARP][2][8];
#pragma unroll
    for (int it = 0; it < WVB_ROWS_PER_WARP; ++it)
#pragma unroll
        for (int u = 0; u < 2; ++u) unpack8(wv[it][u], wf[it][u]);
    __syncthreads();
    for (int c = 0; c < ntp; c += WVB_TCH) {
        float v[32];
#pragma unroll
        for (int tt = 0; tt < WVB_TCH; ++tt) {
            float xf[2][8];
#pragma unroll
            for (int u = 0; u < 2; ++u)
                unpack8(*reinterpret_cast<const uint4*>(xs + (c + tt) * kLatent + 256 * u + 8 * lane), xf[u]);
#pragma unroll
            for (int it = 0; it < WVB_ROWS_PER_WARP; ++it) {
                float acc = 0.0f;
#pragma unroll
                for (int u = 0; u < 2; ++u)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc = fmaf(wf[it][u][j], xf[u][j], acc);
                v[WVB_TCH * it + tt] = acc;
            }
        }
        const float r = xor_transpose_reduce<32>(v, lane);
        const int it = lane / WVB_TCH, t = c + lane % WVB_TCH;
        if (t < nt) out[static_cast<size_t>(t) * outr.ts + h * outr.hs + j0 + it] = r;
    }
}

}  // namespace gemv

cudaError_t launch_wkb_f16(const void* w, const float* q, Rows qr, float* out, Rows outr, int nt,
                           uint32_t flags, cudaStream_t stream) {
    using namespace gemv;
    const int qcat = (flags & M4B_FLAG_QCAT) ? 1 : 0;
    constexpr int rows = kHeads * kLatent;
    constexpr int grid = rows / (WKB_ROWS_PER_WARP * (WKB_THREADS / 32));
    static_assert(kLatent % (WKB_ROWS_PER_WARP * (WKB_THREADS / 32)) == 0, "a CTA spans one head");
    if (nt > 1) {
        const int ntp = (nt + WKB_TCH - 1) / WKB_TCH * WKB_TCH;
        return launch(wkb_f16_batch_kernel, dim3(grid), dim3(WKB_THREADS),
                      static_cast<size_t>(ntp) * kNope * sizeof(__half), stream, flags,
                      static_cast<const __half*>(w), q, qr, out, outr, nt, qcat);
    }
    return launch(wkb_f16_kernel, dim3(grid), dim3(WKB_THREADS), 0, stream, flags,
                  static_cast<const __half*>(w), q, qr, out, outr, nt, qcat);
}

cudaError_t launch_wvb_f16(const void* w, const float* x, Rows xr, float* out, Rows outr, int nt,
                           uint32_t flags, cudaStream_t stream) {
    using namespace gemv;
    constexpr int rows = kHeads * kVHead;
    constexpr int grid = rows / (WVB_ROWS_PER_WARP * (WVB_THREADS / 32));
    static_assert(kVHead % (WVB_ROWS_PER_WARP * (WVB_THREADS / 32)) == 0, "a CTA spans one head");
    if (nt > 1) {
        const int ntp = (nt + WVB_TCH - 1) / WVB_TCH * WVB_TCH;
        const size_t smem = static_cast<size_t>(ntp) * kLatent * sizeof(__half);   // <= 64 KB
        const cudaError_t e = note(cudaFuncSetAttribute(
            wvb_f16_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
            static_cast<int>(kMaxSeqs * kLatent * sizeof(__half))));
        if (e != cudaSuccess) return e;
        return launch(wvb_f16_batch_kernel, dim3(grid), dim3(WVB_THREADS), smem, stream, flags,
                      static_cast<const __half*>(w), x, xr, out, outr, nt);
    }
    return launch(wvb_f16_kernel, dim3(grid), dim3(WVB_THREADS), 0, stream, flags,
                  static_cast<const __half*>(w), x, xr, out, outr, nt);
}

}  // namespace m4b
