// m4b_exchange.cu -- the KV-slab exchange between GPUs, fused into the merge kernels over NVLink.
//
// Long contexts are split into contiguous KV slabs, one per GPU (one process per GPU).  Each GPU
// computes split-K partial records over its slab; the only data that must cross GPUs is one
// merged record per head (32 x 516 values).  Instead of a library collective, the kernel that
// merges this GPU's splits stores its record straight into every peer's receive buffer through
// CUDA IPC peer mappings (NVLink / NVSwitch), and the kernel that consumes the records polls its
// own memory.  No multicast and no TMA reads of peer memory are used.
//
// Flag-in-word records.  Every value travels as one 8-byte word {f32 value, u32 epoch} written
// with a single 64-bit store, so a reader that sees the current epoch in a word also sees that
// word's value: no memory fence, no separate flag and no second NVLink trip.  The cost is 8 bytes
// per 4-byte value, 132 KB per rank and exchange.
//
// Per-GPU buffer (allocated once at set-up, shared by IPC handle):
//   recv[2][world][32][516] u64   records {value, epoch}, double-buffered by epoch parity
//   epoch[32][4] u64              exchanges published so far, one count per (head, 128-column
//                                 block): the CTA that publishes a block reads its count at the
//                                 start and stores the next one at its end, so no CTA waits on
//                                 another's bookkeeping (all counts move in step)
// Every value that changes per call (the epochs, the buffer parity) is read from device memory, so
// the kernels can be captured once in a CUDA graph and replayed.
//
// Reuse of a parity half is safe: a GPU publishes epoch e+2 only after its own consumer of epoch
// e+1 saw every peer's e+1 record, which every peer published after consuming epoch e.
#include <cstring>

#include "m4b_internal.h"
#include "m4b_ptx.cuh"

struct m4b_exchange {
    int world;
    int rank;
    int device;
    char* local;                         // this GPU's buffer
    char* peer[m4b::kMaxWorld];          // every rank's buffer as mapped here (peer[rank] = local)
    bool opened[m4b::kMaxWorld];
    size_t bytes;
};

namespace m4b {
namespace xch {

constexpr size_t kRecordWords = static_cast<size_t>(kHeads) * kPartStride;

constexpr int kColBlocks = kLatent / 128;   // 128-column blocks per head record

struct Layout {
    size_t recv_off, epoch_off, bytes;
};

inline Layout layout(int world) {
    Layout l;
    l.recv_off = 0;
    l.epoch_off = 2 * static_cast<size_t>(world) * kRecordWords * sizeof(uint64_t);
    l.bytes = (l.epoch_off + kHeads * kColBlocks * sizeof(uint64_t) + 255) &
              ~static_cast<size_t>(255);
    return l;
}

// the exchange count of head h's column block y on this GPU
__device__ __forceinline__ volatile uint64_t* epoch_word(char* local, const Layout& L, int h,
                                                         int y) {
    return reinterpret_cast<volatile uint64_t*>(local + L.epoch_off) + h * kColBlocks + y;
}

struct PeerPtrs {
    char* p[kMaxWorld];
};

__device__ __forceinline__ uint64_t* record(char* base, const Layout& L, uint64_t e, int world,
                                            int r, int h) {
    return reinterpret_cast<uint64_t*>(base + L.recv_off) +
           ((e & 1) * world + r) * kRecordWords + static_cast<size_t>(h) * kPartStride;
}

__device__ __forceinline__ void st_word(uint64_t* a, float v, uint32_t e) {
    const uint64_t w = (static_cast<uint64_t>(e) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}

// Poll N words at once until each carries epoch e: every pending word's load is in flight
// together, so once the records are in, the wait costs one L2 round trip instead of one per word
// (per rank).  Bounded: after g_wait_limit cycles (counted from t0) the device status becomes
// TIMEOUT and whatever the words hold is returned.  Words outside `pending` are not read.
template <int N>
__device__ __forceinline__ void ld_words(const uint64_t* const (&a)[N], unsigned pending,
                                         uint32_t e, long long t0, float (&v)[N]) {
    uint64_t w[N];
#pragma unroll
    for (int k = 0; k < N; ++k) w[k] = 0;
    for (;;) {
#pragma unroll
        for (int k = 0; k < N; ++k)
            if ((pending >> k) & 1u)
                asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w[k]) : "l"(a[k]) : "memory");
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (((pending >> k) & 1u) && static_cast<uint32_t>(w[k] >> 32) == e) pending &= ~(1u << k);
        if (pending == 0) break;
        if (wait_expired(t0)) {
            atomicExch(&g_status, DEV_STATUS_TIMEOUT);
            break;
        }
    }
#pragma unroll
    for (int k = 0; k < N; ++k) v[k] = __uint_as_float(static_cast<uint32_t>(w[k]));
}

constexpr int THREADS = 256;

// Merge this GPU's S split records (m4-kqkv.cu:318-338 rule, log2 units) into one unnormalised
// record per head and store it, epoch-tagged, into slot [rank] of every peer's receive buffer.
// grid (32 heads, 4 blocks of 128 latent columns).
__global__ void __launch_bounds__(THREADS)
publish_kernel(const float* __restrict__ part, int S, PeerPtrs peers, char* local, int world,
               int rank, Layout L) {
    extern __shared__ float s_ml[];   // [2][S]
    __shared__ __align__(16) float s_red[THREADS / 32][128];   // written as float4
    __shared__ float s_m[THREADS / 32], s_l[THREADS / 32];
    static_assert(THREADS == kq::CMB_THREADS, "the merge helper assumes the combine's block size");
    pdl_wait();
    const int h = blockIdx.x;
    const int d0 = blockIdx.y * 128;
    const int tid = threadIdx.x;
    const size_t ss = static_cast<size_t>(kHeads) * kPartStride;
    const float* ph = part + static_cast<size_t>(h) * kPartStride;
    volatile uint64_t* ep = epoch_word(local, L, h, blockIdx.y);
    const uint64_t e = *ep + 1;
    float mstar, l, o;
    kq::merge_block_inflight<kLatent>(ph, S, ss, d0, s_ml, s_red, s_m, s_l, mstar, l, o);
    const uint32_t e32 = static_cast<uint32_t>(e);
    if (tid < 128) {
#pragma unroll
        for (int p = 0; p < kMaxWorld; ++p) {   // unrolled: the peer table stays in registers
            if (p >= world) break;
            uint64_t* rec = record(peers.p[p], L, e, world, rank, h);
            st_word(rec + d0 + tid, o, e32);
            if (blockIdx.y == 0 && tid == 0) {
                st_word(rec + kPartM, mstar, e32);
                st_word(rec + kPartL, l, e32);
            }
        }
    }
    // this block's count advances (every thread read it before merge_block_inflight's first
    // barrier; the next kernels on this GPU are ordered after this one by the stream)
    if (tid == 0) *ep = e;
}

// Wait for every rank's record of head h (polling the epoch in each word), merge the `world`
// records, normalise, then apply W_UV to the merged head:
//   out[h][j] = sum_r W_UV[h][j][r] * f16(attn[h][r])          (m4-phase.cu:52-89, ggml F16 mul_mat)
// grid (32 heads, 8 blocks of 16 W_UV rows); each CTA merges its head's 512 columns itself (an L2
// read of world x 4 KB) so the gemv needs no second launch.  The CTA of row block 0 also writes
// the normalised attention row when attn_out is given.
constexpr int GW_ROWS_PER_WARP = 2;
constexpr int GW_ROWS = GW_ROWS_PER_WARP * (THREADS / 32);   // 16 rows per CTA

__global__ void __launch_bounds__(THREADS)
gather_wvb_kernel(char* __restrict__ local, int world, Layout L, const __half* __restrict__ w_uv,
                  float* __restrict__ attn_out, int64_t attn_hs, float* __restrict__ out,
                  int64_t out_hs) {
    __shared__ float s_m[kMaxWorld], s_l[kMaxWorld];
    __shared__ __align__(16) float s_x[kLatent];
    const int h = blockIdx.x;
    const int j0 = blockIdx.y * GW_ROWS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // W_UV rows first: they do not depend on any earlier kernel
    uint4 wv[GW_ROWS_PER_WARP][2];
#pragma unroll
    for (int it = 0; it < GW_ROWS_PER_WARP; ++it)
#pragma unroll
        for (int u = 0; u < 2; ++u)
            wv[it][u] = gemv::ldg_stream(w_uv + (static_cast<size_t>(h) * kVHead + j0 +
                                                 warp * GW_ROWS_PER_WARP + it) * kLatent +
                                         256 * u + 8 * lane);
    pdl_wait();
    const uint64_t e = *epoch_word(local, L, h, 0);   // advanced by the publish just before
    const uint32_t e32 = static_cast<uint32_t>(e);
    const long long t0 = clock64();
    const unsigned all = (1u << world) - 1u;
    if (tid < world) {
        const uint64_t* rec = record(local, L, e, world, tid, h);
        const uint64_t* a[2] = {rec + kPartM, rec + kPartL};
        float ml[2];
        ld_words<2>(a, 3u, e32, t0, ml);
        s_m[tid] = ml[0];
        s_l[tid] = ml[1];
    }
    float v[2][kMaxWorld];
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint64_t* a[kMaxWorld];
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r)
            a[r] = record(local, L, e, world, r < world ? r : 0, h) + tid + c * THREADS;
        ld_words<kMaxWorld>(a, all, e32, t0, v[c]);
    }
    __syncthreads();
    float mstar = -INFINITY;
    for (int r = 0; r < world; ++r) mstar = fmaxf(mstar, s_m[r]);
    float l = 0.0f, o0 = 0.0f, o1 = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
        if (r < world) {
            const float a = (s_m[r] > -INFINITY) ? exp2f(s_m[r] - mstar) : 0.0f;
            l = fmaf(a, s_l[r], l);
            o0 = fmaf(a, v[0][r], o0);
            o1 = fmaf(a, v[1][r], o1);
        }
    }
    const float inv = (mstar > -INFINITY && l > 0.0f) ? 1.0f / l : 0.0f;
    const float x0 = (inv != 0.0f) ? o0 * inv : 0.0f;
    const float x1 = (inv != 0.0f) ? o1 * inv : 0.0f;
    if (attn_out != nullptr && blockIdx.y == 0) {
        attn_out[h * attn_hs + tid] = x0;
        attn_out[h * attn_hs + tid + THREADS] = x1;
    }
    s_x[tid] = gemv::round_f16(x0);
    s_x[tid + THREADS] = gemv::round_f16(x1);
    __syncthreads();
    float xf[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const float4 a = *reinterpret_cast<const float4*>(&s_x[256 * u + 8 * lane]);
        const float4 b = *reinterpret_cast<const float4*>(&s_x[256 * u + 8 * lane + 4]);
        xf[u][0] = a.x; xf[u][1] = a.y; xf[u][2] = a.z; xf[u][3] = a.w;
        xf[u][4] = b.x; xf[u][5] = b.y; xf[u][6] = b.z; xf[u][7] = b.w;
    }
#pragma unroll
    for (int it = 0; it < GW_ROWS_PER_WARP; ++it) {
        float acc = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float wf[8];
            gemv::unpack8(wv[it][u], wf);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fmaf(wf[j], xf[u][j], acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) out[h * out_hs + j0 + warp * GW_ROWS_PER_WARP + it] = acc;
    }
}

// The whole exchange in one launch: per head h and 128-column block (a cluster of the head's
// blocks, as in kqkv_combine_wvb_kernel) -- merge this GPU's S split records (publish_kernel's
// arithmetic), store the block, epoch-tagged, into slot [rank] of every GPU's receive buffer, wait
// (bounded) for every GPU's block of the same exchange, merge those `world` records and normalise
// (gather_wvb_kernel's arithmetic: attn is bit-identical to the two-launch form), then apply the
// block's W_UV slice and add the cluster's partial rows in rank order through distributed shared
// memory.  A block waits only for the same block of the other GPUs, which never waits for anything
// before publishing, so the waits always end.
__global__ void __cluster_dims__(1, kLatent / 128, 1) __launch_bounds__(THREADS)
merge_exchange_wvb_kernel(const float* __restrict__ part, int S, PeerPtrs peers, char* local,
                          int world, int rank, Layout L, const __half* __restrict__ w_uv,
                          float* __restrict__ attn_out, int64_t attn_hs, float* __restrict__ out,
                          int64_t out_hs, int release) {
    namespace cg = cooperative_groups;
    extern __shared__ float s_ml[];   // [2][S]
    __shared__ __align__(16) float s_red[THREADS / 32][128];
    __shared__ float s_m[THREADS / 32], s_l[THREADS / 32];
    __shared__ float s_wm[kMaxWorld], s_wl[kMaxWorld];
    __shared__ __align__(16) __half s_x[128];
    __shared__ float s_part[kVHead];
    const int h = blockIdx.x;
    const int d0 = blockIdx.y * 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hw = lane >> 4, l16 = lane & 15;

    uint4 wv[8];   // W_UV[h][j][d0 .. d0+127], rows 16 * warp .. + 15 (no dependency on earlier kernels)
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int j = 16 * warp + 2 * k + hw;
        wv[k] = kq::ldg_nc_u4(w_uv + (static_cast<size_t>(h) * kVHead + j) * kLatent + d0 + 8 * l16);
    }
    if (release) pdl_launch_dependents();   // M4B_FLAG_EARLY_RELEASE: the next layer's loads may start
    pdl_wait();
    volatile uint64_t* ep = epoch_word(local, L, h, blockIdx.y);
    const uint64_t e = *ep + 1;
    const uint32_t e32 = static_cast<uint32_t>(e);

    // 1. this GPU's record block, stored into every GPU's slot [rank]
    {
        const size_t ss = static_cast<size_t>(kHeads) * kPartStride;
        float mstar, l, o;
        kq::merge_block_inflight<kLatent>(part + static_cast<size_t>(h) * kPartStride, S, ss, d0,
                                          s_ml, s_red, s_m, s_l, mstar, l, o);
        if (tid < 128) {
#pragma unroll
            for (int p = 0; p < kMaxWorld; ++p) {
                if (p >= world) break;
                uint64_t* rec = record(peers.p[p], L, e, world, rank, h);
                st_word(rec + d0 + tid, o, e32);
                if (tid == 0) {   // every block carries m and l: no block waits for another's
                    st_word(rec + kPartM, mstar, e32);
                    st_word(rec + kPartL, l, e32);
                }
            }
        }
    }

    // 2. every GPU's block of this exchange (bounded polls of the epoch in each word)
    const long long t0 = clock64();
    float v[kMaxWorld];
    if (tid < 128) {   // column d0 + tid of every rank's record, all polled together
        const uint64_t* a[kMaxWorld];
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r)
            a[r] = record(local, L, e, world, r < world ? r : 0, h) + d0 + tid;
        ld_words<kMaxWorld>(a, (1u << world) - 1u, e32, t0, v);
    } else if (tid - 128 < world) {   // m and l of rank tid - 128
        const uint64_t* rec = record(local, L, e, world, tid - 128, h);
        const uint64_t* a[2] = {rec + kPartM, rec + kPartL};
        float ml[2];
        ld_words<2>(a, 3u, e32, t0, ml);
        s_wm[tid - 128] = ml[0];
        s_wl[tid - 128] = ml[1];
    }
    __syncthreads();
    if (tid < 128) {
        float mstar = -INFINITY;
        for (int r = 0; r < world; ++r) mstar = fmaxf(mstar, s_wm[r]);
        float l = 0.0f, o = 0.0f;
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r) {
            if (r < world) {
                const float a = (s_wm[r] > -INFINITY) ? exp2f(s_wm[r] - mstar) : 0.0f;
                l = fmaf(a, s_wl[r], l);
                o = fmaf(a, v[r], o);
            }
        }
        const float inv = (mstar > -INFINITY && l > 0.0f) ? 1.0f / l : 0.0f;
        const float x = (inv != 0.0f) ? o * inv : 0.0f;
        if (attn_out != nullptr) attn_out[h * attn_hs + d0 + tid] = x;
        s_x[tid] = __float2half_rn(x);
    }
    __syncthreads();

    // 3. the block's share of W_UV, summed over the cluster in rank order
    float xf[8];
    {
        const uint4 xu = *reinterpret_cast<const uint4*>(s_x + 8 * l16);
        const __half2* x2 = reinterpret_cast<const __half2*>(&xu);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(x2[i]);
            xf[2 * i] = f.x;
            xf[2 * i + 1] = f.y;
        }
    }
    float dots[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const __half2* w2 = reinterpret_cast<const __half2*>(&wv[k]);
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(w2[i]);
            a = fmaf(f.x, xf[2 * i], a);
            a = fmaf(f.y, xf[2 * i + 1], a);
        }
        dots[k] = a;
    }
    float r = kq::butterfly_transpose_sum<8>(dots, lane);
    r += __shfl_xor_sync(0xffffffffu, r, 8);
    if ((l16 & 8) == 0) s_part[16 * warp + 2 * l16 + hw] = r;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0 && tid < kVHead) {
        float o = 0.0f;
#pragma unroll
        for (int b = 0; b < kLatent / 128; ++b) o += cluster.map_shared_rank(s_part, b)[tid];
        out[h * out_hs + tid] = o;
    }
    cluster.sync();

    // 4. this block's count advances (read by every thread before the first barrier)
    if (tid == 0) *ep = e;
}

}  // namespace xch
}  // namespace m4b

using namespace m4b;

extern "C" {

M4B_API int m4b_exchange_create(int world, int rank, m4b_exchange** out) {
    if (!out || world < 1 || world > kMaxWorld || rank < 0 || rank >= world) return M4B_EINVAL;
    *out = nullptr;
    int rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    m4b_exchange* x = new m4b_exchange();
    std::memset(x, 0, sizeof(*x));
    x->world = world;
    x->rank = rank;
    if (cudaGetDevice(&x->device) != cudaSuccess) {
        delete x;
        return M4B_ECUDA;
    }
    const xch::Layout L = xch::layout(world);
    x->bytes = L.bytes;
    void* p = nullptr;
    if (cudaMalloc(&p, L.bytes) != cudaSuccess) {   // set-up time, not on the op path
        delete x;
        return M4B_ECUDA;
    }
    if (cudaMemset(p, 0, L.bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        delete x;
        return M4B_ECUDA;
    }
    x->local = static_cast<char*>(p);
    x->peer[rank] = x->local;
    *out = x;
    return M4B_OK;
}

M4B_API int m4b_exchange_ipc_handle(const m4b_exchange* x, void* handle_out) {
    if (!x || !handle_out) return M4B_EINVAL;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, x->local) != cudaSuccess) return M4B_ECUDA;
    std::memcpy(handle_out, &h, sizeof(h));
    return M4B_OK;
}

M4B_API int m4b_exchange_open(m4b_exchange* x, const void* handles) {
    if (!x || !handles) return M4B_EINVAL;
    const char* hs = static_cast<const char*>(handles);
    for (int r = 0; r < x->world; ++r) {
        if (r == x->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hs + static_cast<size_t>(r) * M4B_IPC_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
            return M4B_ECUDA;
        x->peer[r] = static_cast<char*>(p);
        x->opened[r] = true;
    }
    return M4B_OK;
}

M4B_API int m4b_exchange_open_local(m4b_exchange* x, m4b_exchange* const* all, int n) {
    if (!x || !all || n != x->world || all[x->rank] != x) return M4B_EINVAL;
    for (int r = 0; r < n; ++r)
        if (!all[r] || all[r]->world != x->world || all[r]->rank != r || !all[r]->local)
            return M4B_EINVAL;
    for (int r = 0; r < n; ++r) {
        if (r == x->rank || x->opened[r]) continue;
        if (all[r]->device != x->device) {   // another GPU of this process: direct peer access
            int can = 0;
            if (cudaDeviceCanAccessPeer(&can, x->device, all[r]->device) != cudaSuccess)
                return M4B_ECUDA;
            if (!can) return M4B_EDEVICE;
            int cur = 0;
            if (cudaGetDevice(&cur) != cudaSuccess || cudaSetDevice(x->device) != cudaSuccess)
                return M4B_ECUDA;
            const cudaError_t e = cudaDeviceEnablePeerAccess(all[r]->device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();   // clear it
            cudaSetDevice(cur);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return M4B_ECUDA;
        }
        x->peer[r] = all[r]->local;   // same process: the pointer itself, nothing to unmap
    }
    return M4B_OK;
}

M4B_API int m4b_exchange_detach(m4b_exchange* x) {
    if (!x) return M4B_OK;
    int rc = M4B_OK;
    if (cudaDeviceSynchronize() != cudaSuccess) rc = M4B_ECUDA;   // no launch may still use a peer
    for (int r = 0; r < x->world; ++r) {
        if (x->opened[r] && cudaIpcCloseMemHandle(x->peer[r]) != cudaSuccess) rc = M4B_ECUDA;
        if (r != x->rank) x->peer[r] = nullptr;
        x->opened[r] = false;
    }
    return rc;
}

M4B_API int m4b_exchange_destroy(m4b_exchange* x) {
    if (!x) return M4B_OK;
    int rc = m4b_exchange_detach(x);   // no-op when the caller detached already
    if (x->local && cudaFree(x->local) != cudaSuccess) rc = M4B_ECUDA;
    delete x;
    return rc;
}

M4B_API int m4b_exchange_publish(m4b_exchange* x, const m4b_phase_args* a, m4b_stream_t stream) {
    if (!x || !a) return M4B_EINVAL;
    for (int r = 0; r < x->world; ++r)
        if (!x->peer[r]) return M4B_EINVAL;   // m4b_exchange_open not done
    int rc = check_partials(a->src[1], 0, kGeomBaseline);   // records of the BASELINE geometry
    if (rc != M4B_OK) return rc;
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    xch::PeerPtrs pp;
    for (int r = 0; r < kMaxWorld; ++r) pp.p[r] = r < x->world ? x->peer[r] : nullptr;
    const int S = static_cast<int>(a->src[1].ne[2]);
    const size_t smem = 2 * static_cast<size_t>(S) * sizeof(float);
    if (smem > 48 * 1024) return M4B_EINVAL;
    return status_of(launch(xch::publish_kernel, dim3(kHeads, kLatent / 128), dim3(xch::THREADS),
                            smem, reinterpret_cast<cudaStream_t>(stream), a->flags,
                            static_cast<const float*>(a->src[1].data), S, pp, x->local, x->world, x->rank,
                            xch::layout(x->world)));
}

M4B_API int m4b_exchange_combine_wvb(m4b_exchange* x, const m4b_phase_args* a,
                                     m4b_stream_t stream) {
    if (!x || !a) return M4B_EINVAL;
    if (!x->local) return M4B_EINVAL;
    int geom = 0;
    int rc = check_wuv(a->src[0], &geom);
    if (rc != M4B_OK) return rc;
    if (geom != kGeomBaseline) return M4B_ENOTSUP;   // the exchange carries 516-float records
    rc = check_phase_dst(a->dst);
    if (rc != M4B_OK) return rc;
    float* attn = nullptr;
    int64_t attn_hs = kLatent;
    if (a->src[2].data != nullptr) {
        if (check_attn(a->src[2], kGeomBaseline) != M4B_OK) return M4B_EINVAL;
        attn = static_cast<float*>(a->src[2].data);
        attn_hs = static_cast<int64_t>(a->src[2].nb[2] / 4);
    }
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    return status_of(launch(xch::gather_wvb_kernel, dim3(kHeads, kVHead / xch::GW_ROWS),
                            dim3(xch::THREADS), 0, reinterpret_cast<cudaStream_t>(stream), a->flags,
                            x->local, x->world, xch::layout(x->world),
                            static_cast<const __half*>(a->src[0].data), attn, attn_hs,
                            static_cast<float*>(a->dst.data),
                            static_cast<int64_t>(a->dst.nb[2] / 4)));
}

M4B_API int m4b_exchange_merge_wvb(m4b_exchange* x, const m4b_phase_args* a,
                                   m4b_stream_t stream) {
    if (!x || !a) return M4B_EINVAL;
    for (int r = 0; r < x->world; ++r)
        if (!x->peer[r]) return M4B_EINVAL;   // m4b_exchange_open not done
    int geom = 0;
    int rc = check_wuv(a->src[0], &geom);
    if (rc != M4B_OK) return rc;
    if (geom != kGeomBaseline) return M4B_ENOTSUP;   // the exchange carries 516-float records
    rc = check_partials(a->src[1], kMaxRecords, kGeomBaseline);
    if (rc != M4B_OK) return rc;
    rc = check_phase_dst(a->dst);
    if (rc != M4B_OK) return rc;
    float* attn = nullptr;
    int64_t attn_hs = kLatent;
    if (a->src[2].data != nullptr) {
        if (check_attn(a->src[2], kGeomBaseline) != M4B_OK) return M4B_EINVAL;
        attn = static_cast<float*>(a->src[2].data);
        attn_hs = static_cast<int64_t>(a->src[2].nb[2] / 4);
    }
    rc = device_check(nullptr);
    if (rc != M4B_OK) return rc;
    xch::PeerPtrs pp;
    for (int r = 0; r < kMaxWorld; ++r) pp.p[r] = r < x->world ? x->peer[r] : nullptr;
    const int S = static_cast<int>(a->src[1].ne[2]);
    const size_t smem = 2 * static_cast<size_t>(S) * sizeof(float);
    return status_of(launch(xch::merge_exchange_wvb_kernel, dim3(kHeads, kLatent / 128),
                            dim3(xch::THREADS), smem, reinterpret_cast<cudaStream_t>(stream),
                            a->flags, static_cast<const float*>(a->src[1].data), S, pp, x->local,
                            x->world, x->rank, xch::layout(x->world),
                            static_cast<const __half*>(a->src[0].data), attn, attn_hs,
                            static_cast<float*>(a->dst.data),
                            static_cast<int64_t>(a->dst.nb[2] / 4),
                            (a->flags & M4B_FLAG_EARLY_RELEASE) ? 1 : 0));
}

}  // extern "C"
