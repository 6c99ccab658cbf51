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
               float* __restrict__ out, Rows outr, int nt) {
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

}  // namespace gemv

cudaError_t launch_wkb_f16(const void* w, const float* q, Rows qr, float* out, Rows outr, int nt,
                           uint32_t flags, cudaStream_t stream) {
    using namespace gemv;
    constexpr int rows = kHeads * kLatent;
    constexpr int grid = rows / (WKB_ROWS_PER_WARP * (WKB_THREADS / 32));
    return launch(wkb_f16_kernel, dim3(grid), dim3(WKB_THREADS), 0, stream, flags,
                  static_cast<const __half*>(w), q, qr, out, outr, nt);
}

cudaError_t launch_wvb_f16(const void* w, const float* x, Rows xr, float* out, Rows outr, int nt,
                           uint32_t flags, cudaStream_t stream) {
    using namespace gemv;
    constexpr int rows = kHeads * kVHead;
    constexpr int grid = rows / (WVB_ROWS_PER_WARP * (WVB_THREADS / 32));
    return launch(wvb_f16_kernel, dim3(grid), dim3(WVB_THREADS), 0, stream, flags,
                  static_cast<const __half*>(w), x, xr, out, outr, nt);
}

}  // namespace m4b
