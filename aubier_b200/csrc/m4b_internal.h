// m4b_internal.h -- declarations shared by the M4 kernel translation units (not part of the ABI).
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/m4b.h"

namespace m4b {

// BASELINE geometry (the measured one): 32 heads, q_nope 128, rope 64, latent 512, K row 576,
// V head 128.  Reference constants for the Mistral-Small-4 geometry: engine/m1_layer.h:47-55.
constexpr int kHeads = 32;
constexpr int kNope = 128;
constexpr int kRope = 64;
constexpr int kLatent = 512;
constexpr int kKRow = kLatent + kRope;  // 576
constexpr int kVHead = 128;

// Split-K partial record per (split, head): o[512], m (log2 units), l, 2 pad floats.
// 516 floats = 2064 bytes keeps every record 16-byte aligned.
constexpr int kPartStride = kLatent + 4;
constexpr int kPartM = kLatent;
constexpr int kPartL = kLatent + 1;

constexpr int kTileKeys = 128;   // keys per KQKV tile (the tcgen05 MMA M dimension)
constexpr int kMaxSplits = 148;  // one persistent CTA per B200 SM
constexpr int kMaxRecords = 6144;  // partial records one merge accepts (m and l staged in 48 KB)
constexpr int kMaxWorld = 8;     // GPUs of one node in the KV-slab exchange
constexpr int kMaxSeqs = 64;     // tokens (windows) of one ragged KQKV call

struct KqkvLaunch {
    int latent = kLatent;   // 512 (BASELINE) or 256 (Mistral-Small-4): selects the geometry
    const void* kcache;
    uint64_t kcache_row_bytes;
    int64_t n_kv;
    const float* q;
    int64_t q_head_stride;  // floats
    int64_t q_token_stride; // floats (ragged batch)
    const float* mask;      // nullable; single-window op only
    float kq_scale;
    int splits;             // CTAs
    float* part;            // records: [splits][kHeads][kPartStride], ragged [splits + n_seq - 1]
    uint32_t flags;
    const int32_t* seq_base = nullptr;   // ragged batch: token t attends to cache rows
    const int32_t* seq_len = nullptr;    // [seq_base[t], seq_base[t] + seq_len[t])
    int n_seq = 0;
};

cudaError_t launch_kqkv_partials(const KqkvLaunch& a, cudaStream_t stream);

// out[h][d] = merge over S partial records of latent width `latent`; out head stride in floats.
cudaError_t launch_kqkv_combine(const float* part, int S, int latent, float* out,
                                int64_t out_head_stride, uint32_t flags, cudaStream_t stream);

// Ragged batch: merge each token's records (written by launch_kqkv_partials with seq_base set)
// into out[t * out_ts + h * out_hs + d].
// PHASE selector 2 (f16 W_UV): merge + W_UV in one launch; attn_out may be null.
cudaError_t launch_kqkv_combine_wvb(const float* part, int S, const void* w_uv, float* attn_out,
                                    int64_t attn_hs, float* out, int64_t out_hs, uint32_t flags,
                                    cudaStream_t stream);
cudaError_t launch_kqkv_ragged_combine(const float* part, const int32_t* seq_base,
                                       const int32_t* seq_len, int n_seq, int64_t n_rows,
                                       int splits, int latent, float* out, int64_t out_hs,
                                       int64_t out_ts, uint32_t flags, cudaStream_t stream);

// Merge S partial records into one unnormalised record per head ([32][latent + 4]).
cudaError_t launch_kqkv_merge_records(const float* part, int S, int latent, float* out_records,
                                      uint32_t flags, cudaStream_t stream);

// Per-token activation / output addressing of the gemvs: element (t, h, i) at t*ts + h*hs + i.
struct Rows {
    int64_t hs;   // head stride, floats
    int64_t ts;   // token stride, floats
};

#ifdef __CUDACC__
// M4B_FLAG_QCAT: out[t][h][ooff + c] = q[t][h][qoff + c] for the 64 rope values of head h (the
// graph's concat of q_abs and q_pe), for the tokens t = k, k + nk, ... : the nk CTAs that serve
// head h share its tokens, so each thread moves at most a few values (one L2 round trip).
__device__ __forceinline__ void wkb_concat_rope(const float* __restrict__ q, Rows qr, int qoff,
                                                float* __restrict__ out, Rows outr, int ooff,
                                                int nt, int h, int k, int nk, int nthreads) {
    const int count = k < nt ? (nt - k + nk - 1) / nk : 0;
#pragma unroll 4
    for (int i = threadIdx.x; i < count * 64; i += nthreads) {
        const int t = k + nk * (i >> 6), c = i & 63;
        out[t * outr.ts + h * outr.hs + ooff + c] = q[t * qr.ts + h * qr.hs + qoff + c];
    }
}
#endif

// q_abs[t][h][r] = W_UK[h][r][:] . f16(q[t][h][:128]) for nt tokens; W_UK contiguous f16
// [32][512][128], read once for all tokens.
cudaError_t launch_wkb_f16(const void* w, const float* q, Rows qr, float* out, Rows outr, int nt,
                           uint32_t flags, cudaStream_t stream);

// out[t][h][j] = W_UV[h][j][:] . f16(x[t][h][:512]) for nt tokens; W_UV contiguous f16
// [32][128][512], read once for all tokens.
cudaError_t launch_wvb_f16(const void* w, const float* x, Rows xr, float* out, Rows outr, int nt,
                           uint32_t flags, cudaStream_t stream);

// The last CUDA error a launch of this library hit (m4b_last_cuda_error reads and clears it).
inline std::atomic<int>& last_cuda_error() {
    static std::atomic<int> e{0};
    return e;
}
inline cudaError_t note(cudaError_t e) {
    if (e != cudaSuccess) last_cuda_error().store(static_cast<int>(e));
    return e;
}

// Mistral-Small-4 geometry (engine/m1_layer.h:47-55): Q8_0 gemvs with the reference's Q8_1
// activation numerics.  W_UK Q8_0 [64, 256, 32]; W_UV Q8_0 [256, 128, 32].
cudaError_t launch_wkb_q8(const void* w, const float* q, Rows qr, float* out, Rows outr, int nt,
                          uint32_t flags, cudaStream_t stream);
cudaError_t launch_wvb_q8(const void* w, const float* x, Rows xr, float* out, Rows outr, int nt,
                          uint32_t flags, cudaStream_t stream);

// PHASE selector 0, the KV-write (Mistral geometry): W_kva Q8_0 [4096, 320] . Q8(cur), RMS norm of
// the 256 latent values times norm_w, YaRN rope of the 64 rope values at position pos[0], then
// Kcur (f32, kcur) and its f16 image into cache row kidx[0].
struct KvWriteLaunch {
    const float* cur;           // [4096]
    const void* w;              // Q8_0 [4096, 320]
    const float* norm_w;        // [256]
    void* kcache;               // f16 rows of 320
    int64_t kcache_row_stride;  // halves
    int64_t kcache_rows;
    const int64_t* kidx;        // device
    const int32_t* pos;         // device
    float* kcur;                // [320] out (dst)
    float eps, freq_scale, ext_factor, attn_factor, theta_scale, corr0, corr1;
    uint32_t flags;
    // slab != 0: kidx[0] is a row of the whole cache and kcache holds its rows [slab_base,
    // slab_base + kcache_rows); a row held by another GPU's slab is skipped, not an error
    int slab = 0;
    int64_t slab_base = 0;
};
cudaError_t launch_kvwrite(const KvWriteLaunch& a, cudaStream_t stream);

// Launch helper: plain launch, or with programmatic stream serialisation when PDL is requested.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, uint32_t flags, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (flags & M4B_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return note(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

}  // namespace m4b
