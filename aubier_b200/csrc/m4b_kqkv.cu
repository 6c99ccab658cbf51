// m4b_kqkv.cu -- GGML_OP_M4_KQKV on sm_100a: split-K online-softmax MLA decode attention with
// TMA-staged KV tiles and both contractions on tcgen05 tensor cores, accumulators in TMEM.
//
// What the op computes (the reference's contract, patches/ggml-m4/m4-kqkv.cu:1-37 and the
// unfused graph it replaces, engine/m1_layer.cpp:478-494):
//   s[h][n]  = (K[n] . q[h]) * kq_scale + mask[n]          K[n] = kcache row n, 576 f16
//   out[h]   = sum_n softmax_n(s[h][.]) * V[n]             V[n] = kcache row n, first 512 f16
// All 32 heads share every KV row (MLA's latent cache), so per tile of 128 keys the work is two
// dense products with the heads as the narrow dimension:
//   MMA1  S^T[128 keys x 32 heads]      = Ktile[128 x 576] . Q^T[576 x 32]    (K-major A and B)
//   MMA2  O^T[128-latent block x 32]   += Vtile^T[128 x 128] . P[128 x 32]    (A read MN-major)
// A tcgen05 MMA with N <= 64 costs the same ~65 cycles for M = 64 or 128, so both products use
// M = 128 (128 keys, resp. 128 latent rows, per instruction): ~4.9k tensor cycles per tile.
//
// Shared memory cannot hold a 147 KB tile through its softmax AND the next tile, so the tile is
// read twice: the K pass (all 576 columns, for MMA1) is released as soon as MMA1 consumed it,
// and the V pass (the first 512 columns again, for MMA2) is re-read after the softmax -- from L2,
// where the K pass left it (cache hint evict_last, re-read with evict_first).  HBM still sees
// every KV byte once.  Two rings of 32 KB slots carry the passes: the K ring (3 slots) the K
// passes in tile order, the V ring (2 slots) the V passes, so MMA1 of tile i+1 runs while the
// softmax of tile i works (S and P are double-buffered).
//
// Two MMA-issuing threads.  A tcgen05.mma of M = 128, N = 32 is short (~50 cycles of operand
// reads), and the tensor pipe queues only a few of them: every barrier test, fence and commit of
// a single issuing thread left the pipe idle, which paced the kernel at ~120 cycles per MMA.  So
// MMA1 (S = K . Q) and MMA2 (O += V . P) are issued by two threads, each consuming its own ring
// in order; while one waits or commits, the other's MMAs keep the pipe busy.  Each ring has one
// producer and one consumer, so a slot's barrier is never more than one phase behind its waiter.
// The orderings that one issuing thread used to give by program order are explicit barriers:
// MMA1(t) waits until the softmax of tile t - 2 has read S[t & 1] (p_full), the softmax waits
// for MMA2(t - 2) (o_done[t & 1]) before it rewrites P[t & 1].
//
// CTA = one split (a contiguous run of tiles, balanced as in m4-kqkv.cu:204-218), persistent,
// one per SM.  Ragged batches (several tokens, each attending to its own window [base, base+len)
// of one packed cache -- the engine's per-row mask, m1_layer.cpp:756-773) use the same kernel:
// the tiles of all windows are concatenated and cut into balanced CTA ranges, so a CTA works
// through a short list of segments (one per window it touches), restaging Q and writing one
// partial record at every segment boundary.  The single-token op is the one-segment case.
// Warp roles (384 threads):
//   warp 0      TMA producer of the K ring (from HBM)
//   warp 1      TMEM allocator + the MMA1 issuer (one thread); descriptors are precomputed,
//               each MMA costs one 32-bit add to issue
//   warps 2..9  softmax: two groups of four warps, group g owns heads 16g..16g+15; warp w reads
//               TMEM lanes 32*(w%4).. (one key per thread), does the online softmax in log2 units
//               with a lazy rescale of O (only when a head's max grows by more than 2^15), writes
//               P (f16) for MMA2, and writes the split's (o, m, l) partial record at the end.
//   warp 10     the MMA2 issuer (one thread)
//   warp 11     TMA producer of the V ring (from L2, once the tile's K pass has landed)
// Numerics: q and P are rounded to f16 for the tensor cores -- the same rounding points as the
// reference CPU graph, whose mul_mat converts an F32 src1 to F16 (ggml-cpu.c:1330-1375) -- and
// both products accumulate in f32.
#include <cstddef>
#include <type_traits>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "m4b_internal.h"
#include "m4b_ptx.cuh"

namespace m4b {
namespace kq {

constexpr int H = kHeads;
constexpr int TK = kTileKeys;           // 128 keys per tile
constexpr int CHUNK_BYTES = TK * 128;   // 128 keys x 64 f16 columns = 16 KB, one SW128 TMA box
constexpr int SLOT_BYTES = 2 * CHUNK_BYTES;
// K slots of the five (the rest form the V ring).  Measured at 262,144 keys: 3 K + 2 V slots
// 61-63 us per launch; 4 K + 1 V 100.7 us (each V entry then waits for its L2 refill).
#ifndef M4B_KQ_KSLOTS
#define M4B_KQ_KSLOTS 3
#endif
constexpr int NKSLOT = M4B_KQ_KSLOTS;   // K ring: 32 KB slots, filled from HBM
constexpr int NVSLOT = 5 - NKSLOT;      // V ring: 32 KB slots, refilled from L2
constexpr int NSLOT = NKSLOT + NVSLOT;  // K slots first, then V slots
static_assert(NKSLOT >= 2 && NVSLOT >= 1, "both rings need slots");
constexpr int QCH_BYTES = H * 128;      // 32 heads x 64 columns f16 = 4 KB
constexpr int P_BYTES = 2 * QCH_BYTES;  // 32 heads x 128 keys f16 = 8 KB (double-buffered)
constexpr int CTRL_BYTES = 2048;
constexpr int SEG_BYTES = kMaxSeqs * 32;

// The two head geometries (engine/m1_layer.h:47-55 and the BASELINE shape): latent R = 512 or
// 256, rope 64.  Everything else follows from R: the K pass is the latent chunk pairs plus the
// rope chunk, the V pass the latent pairs; one O^T block of 128 latent rows per pair.
template <int R_>
struct Geo {
    static constexpr int R = R_;
    static constexpr int D = R + kRope;                 // 576 or 320: the KV row
    static constexpr int NCOL = D / 64;                 // 9 or 5 column chunks per key row
    static constexpr int LAT_PAIRS = R / 128;           // 4 or 2
    static constexpr int K_ENTRIES = LAT_PAIRS + 1;     // chunk pairs, then the rope chunk
    static constexpr int V_ENTRIES = LAT_PAIRS;
    static constexpr int PART = R + 4;                  // record: o[R], m, l, 2 pad
    static constexpr int PM = R;
    static constexpr int PL = R + 1;
    static constexpr int OFF_RING = 0;
    static constexpr int OFF_Q = OFF_RING + NSLOT * SLOT_BYTES;
    static constexpr int OFF_P = OFF_Q + NCOL * QCH_BYTES;
    static constexpr int OFF_CTRL = OFF_P + 2 * P_BYTES;
    static constexpr int OFF_SEG = OFF_CTRL + CTRL_BYTES;
    static constexpr int SMEM_BYTES = OFF_SEG + SEG_BYTES + 1024;   // + slack to align to 1 KB
    // S^T x2: cols [0, 64); O^T: LAT_PAIRS blocks of 32 cols from 64 (power-of-two allocation)
    static constexpr int TMEM_COLS = 64 + 32 * LAT_PAIRS <= 128 ? 128 : 256;
    static constexpr int QPER = H * (D / 8) / 256;      // Q units of 8 columns per softmax thread
    static constexpr int QB1 = (QPER + 1) / 2;          // first batch when staging in two
    static_assert(H * (D / 8) % 256 == 0, "Q units must split evenly over the softmax threads");
    static_assert(R % 128 == 0 && (kRope == 64), "latent in 128-column pairs, one rope chunk");
    static_assert(OFF_Q % 1024 == 0 && OFF_P % 1024 == 0 && OFF_CTRL % 16 == 0,
                  "TMA / UMMA operands need 1 KB alignment, vector accesses 16 B");
    static_assert(SMEM_BYTES <= 232448, "exceeds the 227 KB per-CTA shared memory of sm_100");
    static_assert(SMEM_BYTES < (1 << 18), "descriptor low halves assume shared addresses < 256 KB");
    static_assert(PART * 4 % 16 == 0, "records stay 16-byte aligned");
};
using GeoBase = Geo<kLatent>;   // 512
using GeoMistral = Geo<256>;

constexpr int NTHREADS = 384;
constexpr int WARP_KLOAD = 0, WARP_MMA1 = 1, WARP_MMA2 = 10, WARP_VLOAD = 11;
constexpr int TM_S = 0;
constexpr int TM_O = 64;
// log2 units: P = 2^(s - m) stays <= 2^15 (exact in f16, below its 65504 limit) while the running
// max m is stale; a head is rescaled only when a score would exceed that
constexpr float GROW_THRESH = 15.0f;
constexpr float LOG2E = 1.4426950408889634f;

// One run of consecutive tiles of one window, as this CTA processes it.
struct Seg {
    int row0;     // cache row of the segment's first key
    int ntiles;   // tiles in the segment
    int nvalid;   // keys at or after row0 that belong to the window (later keys are masked)
    int seq;      // token index: selects q and, with slot, the output
    int slot;     // partial record index
    int first;    // CTA-local index of the segment's first tile
    int pad[2];
};
static_assert(sizeof(Seg) == 32, "segment table entry");

// Barriers indexed [t & 1] complete one phase per tile of that parity: tile t is phase t >> 1.
struct Ctrl {
    uint64_t kfull[NKSLOT], kempty[NKSLOT];   // K ring: landed / released by MMA1
    uint64_t vfull[NVSLOT], vempty[NVSLOT];   // V ring: landed / released by MMA2
    uint64_t s_full[2];     // MMA1(t) complete: S[t & 1] holds tile t's scores
    uint64_t p_full[2];     // the softmax of tile t wrote P[t & 1] (and has read S[t & 1])
    uint64_t o_done[2];     // MMA2(t) complete: O holds tile t, P[t & 1] may be rewritten
    uint64_t q_full;        // one phase per segment: its token's Q is staged
    uint64_t o_full;        // the MMA2 issuer's last commit
    uint64_t a_fin;         // the MMA1 issuer's last commit
    uint64_t red_full[2];   // per head group, once per tile: the 4 warps' flags / maxima are in
    uint64_t red2_full[2];  // per head group, rare: the exact maxima after a raised flag
    uint64_t redl_full[2];  // per head group: the 4 warps' row sums are in red_l[]
    uint32_t tmem_base;
    int abort_flag;
    int nseg;     // segments of this CTA
    int ntot;     // tiles of this CTA (sum over its segments)
    int k_landed; // tiles whose K pass has landed (MMA1 issuer -> V producer; only grows)
    alignas(16) float red[2][2][4][16];  // [tile parity][group][quadrant][head], read as float4
    alignas(16) float red_l[2][4][16];   // [group][quadrant][head]
    alignas(16) int flag[2][2][4];       // [tile parity][group][quadrant]: a score outgrew the max
};
static_assert(sizeof(Ctrl) <= CTRL_BYTES, "control block too large");
static_assert(offsetof(Ctrl, red) % 16 == 0 && offsetof(Ctrl, red_l) % 16 == 0,
              "reduction buffers are read with 16-byte vector loads");

// 2^x by the special-function unit (ex2.approx: relative error ~2^-22, far below the f16 rounding
// that P gets next; 2^-inf = +0)
__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// A wait whose result is the same in every lane of the warp (the softmax warps run
// warp-collective tcgen05.ld/st and shuffles, which need a converged warp).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    const bool ok = mbar_wait(bar, parity, abort_flag);
    return __all_sync(0xffffffffu, ok);
}

// Column max / sum of a 32(lanes) x 16(values) block held one row per lane: after the
// butterfly each lane holds the reduction of value index (lane >> 1) (lanes 2j, 2j+1 agree).
template <bool kMax>
__device__ __forceinline__ float transpose_reduce16(const float (&in)[16], int lane) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = in[j];
#pragma unroll
    for (int n = 16, off = 16; n > 1; n >>= 1, off >>= 1) {
        const bool upper = (lane & off) != 0;
        const int half = n >> 1;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = upper ? v[i] : v[i + half];
            const float keep = upper ? v[i + half] : v[i];
            const float recv = __shfl_xor_sync(0xffffffffu, send, off);
            v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
        }
    }
    const float r = __shfl_xor_sync(0xffffffffu, v[0], 1);
    return kMax ? fmaxf(v[0], r) : v[0] + r;
}

// Tiles per window for up to 64 windows, two per lane: ts = ceil(len / 128), ps = exclusive prefix
// over the windows in token order, total = all tiles.  A window outside [0, n_rows) counts as
// empty and raises the device status (the host never reads base / len: they may be produced on
// the device, like the reference's kidx / pos, m4-phase.cu:265-267).
struct SeqTiles {
    int ts[2], ps[2], base[2], len[2];
    int total;
};

__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += u;
    }
    return v;
}

__device__ SeqTiles seq_tiles(const int32_t* __restrict__ seq_base,
                              const int32_t* __restrict__ seq_len, int n_seq, int n_rows,
                              int lane) {
    SeqTiles st;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int sq = lane + 32 * k;
        int b = 0, l = 0;
        if (sq < n_seq) {
            b = __ldg(seq_base + sq);
            l = __ldg(seq_len + sq);
            if (b < 0 || l < 0 || static_cast<int64_t>(b) + l > n_rows) {
                bad = true;
                b = 0;
                l = 0;
            }
        }
        st.base[k] = b;
        st.len[k] = l;
        st.ts[k] = (l + TK - 1) / TK;
    }
    const int i0 = warp_incl_scan(st.ts[0], lane);
    const int tot0 = __shfl_sync(0xffffffffu, i0, 31);
    const int i1 = warp_incl_scan(st.ts[1], lane);
    st.total = tot0 + __shfl_sync(0xffffffffu, i1, 31);
    st.ps[0] = i0 - st.ts[0];
    st.ps[1] = tot0 + i1 - st.ts[1];
    if (bad) atomicExch(&g_status, DEV_STATUS_BADSEQ);
    return st;
}

// Balanced cut of T tiles over G CTAs (m4-kqkv.cu:214-218): CTA c owns [lo(c), lo(c) + cnt(c)).
__device__ __forceinline__ int cut_lo(int T, int G, int c) {
    const int b = T / G, r = T % G;
    return c * b + min(c, r);
}
__device__ __forceinline__ int cut_owner(int T, int G, int t) {   // the CTA owning tile t
    const int b = T / G, r = T % G;
    const int big = r * (b + 1);
    return t < big ? t / (b + 1) : r + (t - big) / b;
}

struct KqParams {
    const float* q;
    int64_t q_hs;             // head stride, floats
    int64_t q_ts;             // token stride, floats (ragged)
    const float* mask;        // single-window op only, nullable
    float kq_scale;
    int n_rows;               // cache rows (the single-window op's n_kv)
    float* part;
    uint32_t flags;
    const int32_t* seq_base;  // ragged: per-token window; nullptr for the single-window op
    const int32_t* seq_len;
    int n_seq;
};

template <class G>
__global__ void __launch_bounds__(NTHREADS, 1)
kqkv_partial_kernel(const __grid_constant__ CUtensorMap tmap, const KqParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    Ctrl& C = *reinterpret_cast<Ctrl*>(smem + G::OFF_CTRL);
    Seg* const segs = reinterpret_cast<Seg*>(smem + G::OFF_SEG);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int ncta = gridDim.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < NKSLOT; ++i) {
            mbar_init(&C.kfull[i], 1);
            mbar_init(&C.kempty[i], 1);
        }
        for (int i = 0; i < NVSLOT; ++i) {
            mbar_init(&C.vfull[i], 1);
            mbar_init(&C.vempty[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&C.s_full[b], 1);
            mbar_init(&C.p_full[b], 8);
            mbar_init(&C.o_done[b], 1);
            mbar_init(&C.red_full[b], 4);
            mbar_init(&C.red2_full[b], 4);
            mbar_init(&C.redl_full[b], 4);
        }
        mbar_init(&C.q_full, 256);
        mbar_init(&C.o_full, 1);
        mbar_init(&C.a_fin, 1);
        C.abort_flag = 0;
        C.k_landed = 0;
        fence_mbar_init();
    }
    if (warp == WARP_KLOAD) {
        if (lane == 0) tma_prefetch_desc(&tmap);
        // ---- this CTA's segments
        if (p.seq_base == nullptr) {   // one window: the whole cache, masked by p.mask
            if (lane == 0) {
                const int T = (p.n_rows + TK - 1) / TK;
                const int lo = cut_lo(T, ncta, cta);
                Seg sg = {};
                sg.row0 = lo * TK;
                sg.ntiles = cut_lo(T, ncta, cta + 1) - lo;
                sg.nvalid = p.n_rows - lo * TK;
                sg.seq = 0;
                sg.slot = cta;
                sg.first = 0;
                segs[0] = sg;
                C.nseg = 1;   // written even when empty: every split owns a record
                C.ntot = sg.ntiles;
            }
        } else {
            if (!(p.flags & M4B_FLAG_KV_STATIC)) pdl_wait();   // windows may come from the device
            const SeqTiles st = seq_tiles(p.seq_base, p.seq_len, p.n_seq, p.n_rows, lane);
            const int lo = cut_lo(st.total, ncta, cta), hi = cut_lo(st.total, ncta, cta + 1);
            bool hit[2];
#pragma unroll
            for (int k = 0; k < 2; ++k)
                hit[k] = st.ts[k] > 0 && st.ps[k] < hi && st.ps[k] + st.ts[k] > lo;
            const unsigned b0 = __ballot_sync(0xffffffffu, hit[0]);
            const unsigned b1 = __ballot_sync(0xffffffffu, hit[1]);
            const unsigned below = (1u << lane) - 1u;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                if (!hit[k]) continue;
                const int idx = k == 0 ? __popc(b0 & below) : __popc(b0) + __popc(b1 & below);
                const int a = max(lo, st.ps[k]), e = min(hi, st.ps[k] + st.ts[k]);
                const int j0 = a - st.ps[k];
                Seg sg = {};
                sg.row0 = st.base[k] + j0 * TK;
                sg.ntiles = e - a;
                sg.nvalid = st.len[k] - j0 * TK;
                sg.seq = lane + 32 * k;
                sg.slot = cta + sg.seq;
                sg.first = a - lo;
                segs[idx] = sg;
            }
            if (lane == 0) {
                C.nseg = __popc(b0) + __popc(b1);
                C.ntot = hi - lo;
            }
        }
    }
    if (warp == WARP_MMA1) {
        tmem_alloc(&C.tmem_base, G::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = C.tmem_base;
    volatile int* abort_flag = &C.abort_flag;
    const int nseg = C.nseg;
    const int NT = C.ntot;
    // segment holding CTA-local tile t, advancing a cursor (tiles are visited in order)
    auto seg_of = [&](int t, int& g) -> const Seg& {
        while (t >= segs[g].first + segs[g].ntiles) ++g;
        return segs[g];
    };

    if (warp == WARP_KLOAD || warp == WARP_VLOAD) {
        // ------------------------------------------------------------------ TMA producers
        // warp 0 feeds the K ring with every tile's K pass from HBM (kept in L2 for the V pass);
        // warp 11 feeds the V ring with tile t's V pass once MMA1 has seen its K pass land, so
        // the re-read hits L2.  Each is the only producer of its ring and fills it in order.
        if (lane == 0 && NT > 0) {
            const bool kring = warp == WARP_KLOAD;
            if (!(p.flags & M4B_FLAG_KV_STATIC)) pdl_wait();
            const uint64_t pol = kring ? l2_policy_evict_last()     // K pass: V is re-read soon
                                       : l2_policy_evict_first();   // V pass: last use
            uint64_t* const full = kring ? C.kfull : C.vfull;
            uint64_t* const empty = kring ? C.kempty : C.vempty;
            const int nslot = kring ? NKSLOT : NVSLOT;
            const int nent = kring ? G::K_ENTRIES : G::V_ENTRIES;
            uint8_t* const ring = smem + G::OFF_RING + (kring ? 0 : NKSLOT * SLOT_BYTES);
            int slot = 0, phase = 0, issued = 0, g = 0;
            bool ok = true;
            for (int t = 0; t < NT && ok; ++t) {
                const Seg& sg = seg_of(t, g);
                const int key0 = sg.row0 + (t - sg.first) * TK;
                if (!kring) ok = count_wait(&C.k_landed, t + 1, abort_flag);
                // entry e: chunks 2e and 2e + 1 (columns 128e ..), or the rope chunk alone
                for (int e = 0; e < nent && ok; ++e) {
                    ok = mbar_wait(&empty[slot], phase ^ 1, abort_flag);
                    if (!ok) break;
                    const bool two = e < G::LAT_PAIRS;
                    mbar_arrive_expect_tx(&full[slot], two ? SLOT_BYTES : CHUNK_BYTES);
                    uint8_t* dst = ring + slot * SLOT_BYTES;
                    tma_load_2d(dst, &tmap, 128 * e, key0, &full[slot], pol);
                    if (two) tma_load_2d(dst + CHUNK_BYTES, &tmap, 128 * e + 64, key0, &full[slot], pol);
                    ++issued;
                    if (++slot == nslot) {
                        slot = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag) {
                // let this CTA's own copies land before its shared memory is released: the
                // latest use of every slot
                for (int sl = 0; sl < nslot; ++sl) {
                    const int n = issued > sl ? (issued - sl + nslot - 1) / nslot : 0;
                    if (n > 0) mbar_drain(&full[sl], (n - 1) & 1);
                }
            }
        }
    } else if (warp == WARP_MMA1 || warp == WARP_MMA2) {
        // ------------------------------------------------------------------ MMA issuers
        if (lane == 0) {
            constexpr uint32_t hi = sdesc_sw128_hi(1024);   // SBO = 8 rows x 128 B
            constexpr uint32_t U_CHUNK = CHUNK_BYTES >> 4, U_SLOT = SLOT_BYTES >> 4;
            constexpr uint32_t U_QCH = QCH_BYTES >> 4, U_P = P_BYTES >> 4;
            int slot = 0, phase = 0, g = 0;
            bool ok = true;
            if (warp == WARP_MMA1) {
                // MMA1 of tile t into S[t & 1]: S^T[keys x heads] = K . Q^T, both K-major
                constexpr uint32_t idesc_s = idesc_f16_f32(128, 32, false, false);
                const uint32_t lo_ring = sdesc_sw128_lo(smem_u32(smem + G::OFF_RING), 16);
                const uint32_t lo_q = sdesc_sw128_lo(smem_u32(smem + G::OFF_Q), 16);
                for (int t = 0; t < NT && ok; ++t) {
                    const Seg& sg = seg_of(t, g);
                    // a segment's first tile needs its token's Q (segment g is q_full's phase g)
                    if (t == sg.first) ok = mbar_wait(&C.q_full, g & 1, abort_flag);
                    // S[t & 1] is free once the softmax of tile t - 2 has read it: it wrote P(t - 2)
                    if (ok && t >= 2) ok = mbar_wait(&C.p_full[t & 1], ((t - 2) >> 1) & 1, abort_flag);
                    const uint32_t dS = tmem + TM_S + 32 * (t & 1);
                    for (int e = 0; e < G::K_ENTRIES && ok; ++e) {
                        ok = mbar_wait(&C.kfull[slot], phase, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t a = lo_ring + slot * U_SLOT;
                        const uint32_t b = lo_q + 2 * e * U_QCH;
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            if (hf == 1 && e == G::LAT_PAIRS) break;
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)
                                mma_f16(dS, sdesc_join(a + hf * U_CHUNK + 2 * kk, hi),
                                        sdesc_join(b + hf * U_QCH + 2 * kk, hi), idesc_s,
                                        (e | hf | kk) != 0 ? 1u : 0u);
                        }
                        mma_commit(&C.kempty[slot]);
                        if (++slot == NKSLOT) {
                            slot = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit(&C.s_full[t & 1]);
                    *reinterpret_cast<volatile int*>(&C.k_landed) = t + 1;   // its V pass may go
                }
                // every MMA1 of this thread has completed before the CTA frees TMEM
                mma_commit(&C.a_fin);
                mbar_drain(&C.a_fin, 0);
            } else {
                // MMA2 of tile i: O^T[latent block x heads] += V^T . P, V read MN-major from the
                // V pass itself; the first tile of a segment starts a fresh accumulator
                constexpr uint32_t idesc_o = idesc_f16_f32(128, 32, true, false);
                const uint32_t lo_ring = sdesc_sw128_lo(smem_u32(smem + G::OFF_RING + NKSLOT * SLOT_BYTES),
                                                        CHUNK_BYTES);
                const uint32_t lo_p = sdesc_sw128_lo(smem_u32(smem + G::OFF_P), 16);
                for (int i = 0; i < NT && ok; ++i) {
                    const Seg& sg = seg_of(i, g);
                    ok = mbar_wait(&C.p_full[i & 1], (i >> 1) & 1, abort_flag);
                    if (!ok) break;
                    const uint32_t p0 = lo_p + (i & 1) * U_P;
                    const uint32_t acc0 = i != sg.first ? 1u : 0u;
                    for (int b = 0; b < G::V_ENTRIES && ok; ++b) {
                        ok = mbar_wait(&C.vfull[slot], phase, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t a0 = lo_ring + slot * U_SLOT;
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks)
                            mma_f16(tmem + TM_O + 32 * b, sdesc_join(a0 + ks * (2048 >> 4), hi),
                                    sdesc_join(p0 + (ks >> 2) * U_QCH + 2 * (ks & 3), hi), idesc_o,
                                    ks > 0 ? 1u : acc0);
                        mma_commit(&C.vempty[slot]);
                        if (++slot == NVSLOT) {
                            slot = 0;
                            phase ^= 1;
                        }
                    }
                    if (!ok) break;
                    mma_commit(&C.o_done[i & 1]);
                }
                mma_commit(&C.o_full);
                mbar_drain(&C.o_full, 0);
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax warps
        const int sw = warp - 2;       // 0..7
        const int grp = sw >> 2;       // heads 16*grp .. 16*grp+15
        const int quad = warp & 3;     // TMEM lane quadrant this warp may access
        const int key_in_tile = quad * 32 + lane;   // M = 128 layout: lane = row
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;

        // Stage one token's Q (f32 -> f16, round to nearest even) into the K-major SW128 layout.
        // Each thread converts 9 units of 8 floats with all loads issued before their first use:
        // one L2 round trip instead of nine dependent ones, which matters because the ring has HBM
        // saturated by then (nine round trips measured ~6.6 us, stalling the first MMA).  At a
        // window boundary inside the tile loop, where the softmax state is live, the loads go in
        // two batches (5 + 4 units at BASELINE) to stay within the 168 registers that 12 warps per SM allow
        // (3 warps share one 16K-register sub-partition).
        auto stage_q = [&](const float* qs, bool one_batch) {
            constexpr int D = G::D;
            constexpr int PER = G::QPER;         // 9 (BASELINE) or 5 units of 8 columns
            const int tid = threadIdx.x - 64;
            const bool vec = ((reinterpret_cast<uintptr_t>(qs) |
                               static_cast<uintptr_t>(p.q_hs * 4)) & 15) == 0;   // uniform
            auto batch = [&](auto k0_c, auto nk_c) {
                constexpr int K0 = decltype(k0_c)::value, NK = decltype(nk_c)::value;
                float4 v[NK][2];
#pragma unroll
                for (int k = 0; k < NK; ++k) {
                    const int u = tid + 256 * (K0 + k);
                    const float* src = qs + (u / (D / 8)) * p.q_hs + (u % (D / 8)) * 8;
                    if (vec) {
                        v[k][0] = reinterpret_cast<const float4*>(src)[0];
                        v[k][1] = reinterpret_cast<const float4*>(src)[1];
                    } else {
                        v[k][0] = make_float4(src[0], src[1], src[2], src[3]);
                        v[k][1] = make_float4(src[4], src[5], src[6], src[7]);
                    }
                }
#pragma unroll
                for (int k = 0; k < NK; ++k) {
                    const int u = tid + 256 * (K0 + k);
                    const int h = u / (D / 8);
                    const int col = (u % (D / 8)) * 8;
                    uint4 pk;
                    pk.x = pack_half2(v[k][0].x, v[k][0].y);
                    pk.y = pack_half2(v[k][0].z, v[k][0].w);
                    pk.z = pack_half2(v[k][1].x, v[k][1].y);
                    pk.w = pack_half2(v[k][1].z, v[k][1].w);
                    const int chunk = col >> 6;
                    const int unit = (col & 63) >> 3;
                    *reinterpret_cast<uint4*>(smem + G::OFF_Q + chunk * QCH_BYTES + h * 128 +
                                              ((unit ^ (h & 7)) << 4)) = pk;
                }
            };
            if (one_batch) {
                batch(std::integral_constant<int, 0>{}, std::integral_constant<int, PER>{});
            } else {
                batch(std::integral_constant<int, 0>{}, std::integral_constant<int, G::QB1>{});
                batch(std::integral_constant<int, G::QB1>{},
                      std::integral_constant<int, PER - G::QB1>{});
            }
            fence_proxy_async_smem();
            mbar_arrive(&C.q_full);
        };
        pdl_wait();
        if (NT > 0) stage_q(p.q + segs[0].seq * p.q_ts, true);

        // P destination of this thread's key: column key_in_tile of the 32 head rows, K-major,
        // as two 64-key chunks of 4 KB
        uint8_t* const prow0 = smem + G::OFF_P + (key_in_tile >> 6) * QCH_BYTES + (key_in_tile & 7) * 2;
        const int punit = (key_in_tile & 63) >> 3;

        float m_run[16], l_part[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            m_run[j] = -INFINITY;
            l_part[j] = 0.0f;
        }
        bool ok = true;
        int nflush = 0;
        int nrare = 0;   // red2_full phases used (uniform in the group)
        // ---- a segment's partial record (o[512], m, l) per head; o is read from TMEM once the
        // segment's last MMA2 is complete (bar, parity)
        auto flush = [&](const Seg& sg, uint64_t* bar, uint32_t parity) {
            float* prec = p.part + static_cast<size_t>(sg.slot) * H * G::PART;
            const float lsum = transpose_reduce16<false>(l_part, lane);
            if (ok) {
                if ((lane & 1) == 0) C.red_l[grp][quad][lane >> 1] = lsum;
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.redl_full[grp]);
                ok = warp_wait(&C.redl_full[grp], nflush & 1, abort_flag);
            }
            ++nflush;
            if (ok && quad == 0 && lane < 16) {
                const int h = 16 * grp + lane;
                const float l = C.red_l[grp][0][lane] + C.red_l[grp][1][lane] +
                                C.red_l[grp][2][lane] + C.red_l[grp][3][lane];
                float m = -INFINITY;
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (lane == j) m = m_run[j];
                prec[h * G::PART + G::PM] = m;
                prec[h * G::PART + G::PL] = l;
            }
            if (!ok) return;
            ok = warp_wait(bar, parity, abort_flag);
            if (!ok) return;
            tc_fence_after();
#pragma unroll
            for (int b = 0; b < G::LAT_PAIRS; ++b) {
                float o[16];
                if (sg.ntiles > 0) {
                    tmem_ld16(tmem + lane_off + TM_O + 32 * b + 16 * grp, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) o[j] = 0.0f;   // an empty split: o = 0
                }
                const int d = 128 * b + quad * 32 + lane;   // M = 128 layout: every lane is a row
#pragma unroll
                for (int j = 0; j < 16; ++j) prec[(16 * grp + j) * G::PART + d] = o[j];
            }
        };

        int g = 0;
        for (int i = 0; i < NT; ++i) {
            const Seg& sg = seg_of(i, g);
            const int kl = (i - sg.first) * TK + key_in_tile;   // key index from the segment start
            const bool valid = kl < sg.nvalid;
            float mv = 0.0f;
            if (valid && p.mask != nullptr) mv = __ldg(p.mask + sg.row0 + kl);
            ok = warp_wait(&C.s_full[i & 1], (i >> 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            float s[16];
            tmem_ld16(tmem + lane_off + TM_S + 32 * (i & 1) + 16 * grp, s);
            tmem_wait_ld();
            // MMA1(i) is complete, so Q is free: the next segment's token goes in now
            const bool seg_end = (i == sg.first + sg.ntiles - 1);
            if (seg_end && g + 1 < nseg) stage_q(p.q + segs[g + 1].seq * p.q_ts, false);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                float t = s[j] * p.kq_scale;   // soft_max_ext: scale, then add the mask
                t = t + mv;
                s[j] = valid ? t * LOG2E : -INFINITY;
            }
            // The running max m_run is shared by the group's 4 warps (their keys feed one O per
            // head).  It only has to bound the scores, not track them: P = 2^(s - m_run) is exact
            // in f16 up to 2^15.  So a tile normally costs one vote per warp ("does any score exceed
            // m_run + 15?"); the exact maxima are exchanged, and m_run raised, only on a head's
            // first keys or when a vote is raised (rare) -- shared-memory and shuffle traffic queue
            // behind the tensor core's operand reads, and this keeps it off the critical path.
            bool fresh = false;
#pragma unroll
            for (int j = 0; j < 16; ++j) fresh |= (m_run[j] == -INFINITY);   // uniform in the group
            bool exchange = fresh;
            if (!fresh) {
                bool big = false;
#pragma unroll
                for (int j = 0; j < 16; ++j) big |= (s[j] - m_run[j] > GROW_THRESH);
                const bool wbig = __any_sync(0xffffffffu, big);
                if (lane == 0) C.flag[i & 1][grp][quad] = wbig ? 1 : 0;
                __syncwarp();
                if (lane == 0) mbar_arrive(&C.red_full[grp]);
                ok = warp_wait(&C.red_full[grp], i & 1, abort_flag);
                if (!ok) break;
                const int4 f = *reinterpret_cast<const int4*>(&C.flag[i & 1][grp][0]);
                exchange = (f.x | f.y | f.z | f.w) != 0;
            }
            bool need = false;
            float alpha[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) alpha[j] = 1.0f;
            if (exchange) {
                const float wmax = transpose_reduce16<true>(s, lane);
                if ((lane & 1) == 0) C.red[i & 1][grp][quad][lane >> 1] = wmax;
                __syncwarp();
                uint64_t* bar = fresh ? &C.red_full[grp] : &C.red2_full[grp];
                const uint32_t par = fresh ? (i & 1) : (nrare & 1);
                if (lane == 0) mbar_arrive(bar);
                ok = warp_wait(bar, par, abort_flag);
                if (!ok) break;
                if (!fresh) ++nrare;
                // lane j < 16 combines head j's four quadrant maxima, then all lanes get all 16
                float hm = -INFINITY;
                if (lane < 16) {
                    const float* r = &C.red[i & 1][grp][0][lane];
                    hm = fmaxf(fmaxf(r[0], r[16]), fmaxf(r[32], r[48]));
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float tmax = __shfl_sync(0xffffffffu, hm, j);
                    const float mn = fmaxf(m_run[j], tmax);
                    if (m_run[j] == -INFINITY) {
                        m_run[j] = mn;          // nothing accumulated yet for this head
                    } else if (mn > m_run[j]) {
                        alpha[j] = exp2f(m_run[j] - mn);
                        m_run[j] = mn;
                        need = true;
                    }
                }
            }
            // P[i & 1] is free once MMA2(i - 2) has completed.  o_done[i & 1] is then at most
            // one phase behind (the wait of tile i - 2 saw tile i - 4's phase) and cannot be
            // ahead (tile i's phase needs this P), so the parity wait is exact; the same holds
            // for the waits on o_done below.
            if (i >= 2) {
                ok = warp_wait(&C.o_done[i & 1], ((i - 2) >> 1) & 1, abort_flag);
                if (!ok) break;
            }
            if (need) {   // uniform across the group: every thread computed the same maxima
                // O holds the sum through tile i-1 (same segment): wait for MMA2(i-1)
                ok = warp_wait(&C.o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < 16; ++j) l_part[j] *= alpha[j];
#pragma unroll
                for (int b = 0; b < G::LAT_PAIRS; ++b) {
                    float o[16];
                    const uint32_t ta = tmem + lane_off + TM_O + 32 * b + 16 * grp;
                    tmem_ld16(ta, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) o[j] *= alpha[j];
                    tmem_st16(ta, o);
                }
                tmem_wait_st();
            }
            uint8_t* const prow = prow0 + (i & 1) * P_BYTES;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                // masked key: 2^-inf = 0; a head with no valid key yet has m_run = -inf and the
                // difference NaN, which fmaxf also turns into -inf
                const float pv = ex2_fast(fmaxf(s[j] - m_run[j], -INFINITY));
                l_part[j] += pv;
                const int h = 16 * grp + j;
                *reinterpret_cast<__half*>(prow + h * 128 + ((punit ^ (h & 7)) << 4)) =
                    __float2half_rn(pv);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&C.p_full[i & 1]);
            if (seg_end && g + 1 < nseg) {
                // a segment other than the last ends here: write its record once MMA2(i) is
                // done (the next segment's MMA2 waits for P(i+1), written after this).  MMA2(i)
                // completing means the MMA2 thread's earlier MMAs have completed too.
                flush(sg, &C.o_done[i & 1], (i >> 1) & 1);
                if (!ok) break;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    m_run[j] = -INFINITY;
                    l_part[j] = 0.0f;
                }
            }
        }
        // ---- the last segment's record (every split of the single-window op has one)
        if (ok && nseg > 0) flush(segs[nseg - 1], &C.o_full, 0);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == WARP_MMA1) {
        tc_fence_after();
        tmem_dealloc(tmem, G::TMEM_COLS);
    }
}

// Merge S partial records per head with the online-softmax rule of m4-kqkv.cu:318-338 (log2
// units here): m* = max m_s; a_s = 2^(m_s - m*); out = sum a_s o_s / sum a_s l_s; a head whose
// every split is fully masked gives 0.  CTA = (head, 128 latent columns); the 8 warps split the
// records, each lane accumulates 4 columns with 16-byte loads, one reduction through shared
// memory at the end.  S may exceed one GPU's split count (records gathered from other GPUs).
constexpr int CMB_THREADS = 256;

// Records of latent width R (o[R], m, l, 2 pad).  ph = head h's record of the first split;
// records are ss floats apart; blockIdx.y selects 128 of the R columns.
// record_out == 0: out[d] = merged, normalised attention (out = the head's output row).
// record_out != 0: out = the head's record [kPartStride]: the merged, unnormalised record
// (o = sum a_s o_s, m = m*, l = sum a_s l_s) -- the form that is exchanged between GPUs.
constexpr int CWV_RB = 19;   // records per warp in flight: 8 warps x 19 >= 148 splits

__device__ __forceinline__ uint4 ldg_nc_u4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

template <int N>
__device__ __forceinline__ float butterfly_transpose_sum(float (&v)[N], int lane) {
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
    return v[0];   // lane L: the sum over its xor group of value index (L & (N - 1))
}

// Merge one head's S records over the 128 columns at d0 with every record load of a warp in flight
// at once: merge_head's rule, order and rounding (m4-kqkv.cu:318-338; log2 units).  ph: the head's
// first record, ss: the record stride in floats, s_ml: 2 * S floats of shared memory.  On return
// every thread has mstar and l; threads tid < 128 have the unnormalised column sum o of column
// d0 + tid.  Called by all CMB_THREADS threads.
template <int R, int RB = CWV_RB>
__device__ __forceinline__ void merge_block_inflight(const float* __restrict__ ph, int S, size_t ss,
                                                     int d0, float* s_ml,
                                                     float (*s_red)[128], float* s_m, float* s_l,
                                                     float& mstar, float& l, float& o) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float4 ov[RB];
    auto load_records = [&](int sb) {
#pragma unroll
        for (int k = 0; k < RB; ++k) {
            const int s = sb + warp + 8 * k;
            ov[k] = s < S ? __ldg(reinterpret_cast<const float4*>(ph + s * ss + d0 + 4 * lane))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    load_records(0);
    float* s_ms = s_ml;
    float* s_ls = s_ml + S;
    float m = -INFINITY;
    for (int s = tid; s < S; s += CMB_THREADS) {
        const float ms = __ldg(ph + s * ss + R);
        s_ms[s] = ms;
        s_ls[s] = __ldg(ph + s * ss + (R + 1));
        m = fmaxf(m, ms);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_m[warp] = m;
    __syncthreads();
    mstar = s_m[0];
#pragma unroll
    for (int w = 1; w < CMB_THREADS / 32; ++w) mstar = fmaxf(mstar, s_m[w]);
    float lsum = 0.0f;
    for (int s = tid; s < S; s += CMB_THREADS) {
        const float ms = s_ms[s];
        const float a = (ms > -INFINITY) ? exp2f(ms - mstar) : 0.0f;
        s_ms[s] = a;   // alpha
        lsum += a * s_ls[s];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    if (lane == 0) s_l[warp] = lsum;
    __syncthreads();

    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sb = 0;;) {
#pragma unroll
        for (int k = 0; k < RB; ++k) {
            const int s = sb + warp + 8 * k;
            if (s < S) {
                const float a = s_ms[s];
                acc.x = fmaf(a, ov[k].x, acc.x);
                acc.y = fmaf(a, ov[k].y, acc.y);
                acc.z = fmaf(a, ov[k].z, acc.z);
                acc.w = fmaf(a, ov[k].w, acc.w);
            }
        }
        sb += 8 * RB;
        if (sb >= S) break;
        load_records(sb);
    }
    *reinterpret_cast<float4*>(&s_red[warp][4 * lane]) = acc;
    __syncthreads();
    o = 0.0f;
    l = 0.0f;
#pragma unroll
    for (int w = 0; w < CMB_THREADS / 32; ++w) l += s_l[w];
    if (tid < 128) {
#pragma unroll
        for (int w = 0; w < CMB_THREADS / 32; ++w) o += s_red[w][tid];
    }
}

template <int R, int RB = CWV_RB>
__device__ __forceinline__ void merge_head(const float* __restrict__ ph, int S, size_t ss,
                                           float* __restrict__ out, int record_out,
                                           float* s_ml) {
    __shared__ __align__(16) float s_red[CMB_THREADS / 32][128];   // written as float4
    __shared__ float s_m[CMB_THREADS / 32], s_l[CMB_THREADS / 32];
    const int d0 = blockIdx.y * 128;
    const int tid = threadIdx.x;
    float mstar, l, o;
    merge_block_inflight<R, RB>(ph, S, ss, d0, s_ml, s_red, s_m, s_l, mstar, l, o);
    if (tid < 128) {
        if (record_out) {
            out[d0 + tid] = o;
            if (blockIdx.y == 0 && tid == 0) {
                out[R] = mstar;
                out[(R + 1)] = l;
                out[R + 2] = 0.0f;
                out[R + 3] = 0.0f;
            }
        } else {
            out[d0 + tid] = (mstar > -INFINITY) ? o / l : 0.0f;
        }
    }
}

// grid (32 heads, R / 128 blocks of 128 columns).  record_out: see merge_head; out_hs = the
// output's head stride in floats (R + 4 for records).
template <int R>
__global__ void __launch_bounds__(CMB_THREADS)
kqkv_combine_kernel(const float* __restrict__ part, int S, float* __restrict__ out, int64_t out_hs,
                    int record_out) {
    extern __shared__ float s_ml[];   // [2][S]
    pdl_wait();
    const int h = blockIdx.x;
    merge_head<R>(part + static_cast<size_t>(h) * (R + 4), S, static_cast<size_t>(H) * (R + 4),
                  out + h * out_hs, record_out, s_ml);
}

// PHASE selector 2 in one launch: the LSE merge of one head's 128-column block (merge_head's
// arithmetic and order, so attn is bit-identical to kqkv_combine_kernel's) followed by that block's
// share of W_UV: out[h][j] = sum over the R / 128 column blocks of sum_r W_UV[h][j][r] * f16(attn[h][r]).
// The blocks of a head form a thread-block cluster; rank 0 adds the blocks' partial rows in rank order
// through distributed shared memory (plain loads, no multicast), so the result is deterministic.  All
// record loads of a warp (m, l, and up to RB records' 128 columns) are issued before the first use:
// one L2 round trip where the two-launch form waited on several.  The block's W_UV slice (32 KB) is
// loaded before griddepcontrol.wait, overlapping the KQKV tail.  Compared with the two launches it
// replaces, only the order of W_UV's additions differs (per block, then across blocks).
template <int R>
__global__ void __cluster_dims__(1, R / 128, 1) __launch_bounds__(CMB_THREADS)
kqkv_combine_wvb_kernel(const float* __restrict__ part, int S, const __half* __restrict__ w_uv,
                        float* __restrict__ attn_out, int64_t attn_hs, float* __restrict__ out,
                        int64_t out_hs, int release) {
    namespace cg = cooperative_groups;
    extern __shared__ float s_ml[];   // [2][S]: m then alpha, l
    __shared__ __align__(16) float s_red[CMB_THREADS / 32][128];
    __shared__ float s_m[CMB_THREADS / 32], s_l[CMB_THREADS / 32];
    __shared__ __align__(16) __half s_x[128];
    __shared__ float s_part[kVHead];
    const int h = blockIdx.x;
    const int d0 = blockIdx.y * 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t ss = static_cast<size_t>(kHeads) * (R + 4);
    const float* ph = part + static_cast<size_t>(h) * (R + 4);

    // W_UV[h][j][d0 .. d0+127]: warp w holds rows 16w .. 16w+15, a half-warp one row per step
    const int hw = lane >> 4, l16 = lane & 15;
    uint4 wv[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int j = 16 * warp + 2 * k + hw;
        wv[k] = ldg_nc_u4(w_uv + (static_cast<size_t>(h) * kVHead + j) * R + d0 + 8 * l16);
    }
    if (release) pdl_launch_dependents();   // M4B_FLAG_EARLY_RELEASE: the next layer's loads may start
    pdl_wait();

    float mstar, l, o;
    merge_block_inflight<R>(ph, S, ss, d0, s_ml, s_red, s_m, s_l, mstar, l, o);
    if (tid < 128) {
        const float at = (mstar > -INFINITY) ? o / l : 0.0f;
        if (attn_out != nullptr) attn_out[h * attn_hs + d0 + tid] = at;
        s_x[tid] = __float2half_rn(at);
    }
    __syncthreads();

    // this block's share of W_UV: 8 rows per half-warp, a lane's 8 columns, one transpose-sum
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
    float r = butterfly_transpose_sum<8>(dots, lane);   // lanes 8 apart hold the two half-sums
    r += __shfl_xor_sync(0xffffffffu, r, 8);
    if ((l16 & 8) == 0) s_part[16 * warp + 2 * l16 + hw] = r;

    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (cluster.block_rank() == 0 && tid < kVHead) {
        float o = 0.0f;
#pragma unroll
        for (int b = 0; b < R / 128; ++b) o += cluster.map_shared_rank(s_part, b)[tid];
        out[h * out_hs + tid] = o;
    }
    cluster.sync();   // the other blocks' shared memory stays alive until rank 0 has read it
}

// Ragged batch: grid (32 heads, R / 128 column blocks, n_seq tokens).  Token t's window covers tiles
// [ps, ps + ts) of the concatenation; the CTAs owning them wrote their records for t at slots
// c + t (kqkv_partial_kernel), so the records to merge are the contiguous slots
// [c_first + t, c_last + t].  An empty window gives 0 (m4-kqkv.cu:337).
template <int R>
__global__ void __launch_bounds__(CMB_THREADS)
kqkv_ragged_combine_kernel(const float* __restrict__ part, const int32_t* __restrict__ seq_base,
                           const int32_t* __restrict__ seq_len, int n_seq, int n_rows, int G,
                           float* __restrict__ out, int64_t out_hs, int64_t out_ts) {
    __shared__ float s_ml[2 * kMaxSplits];
    __shared__ int s_first, s_count;
    pdl_wait();
    const int h = blockIdx.x;
    const int t = blockIdx.z;
    if (threadIdx.x < 32) {
        const SeqTiles st = seq_tiles(seq_base, seq_len, n_seq, n_rows, threadIdx.x);
        const int k = t >> 5;
        const int ts = __shfl_sync(0xffffffffu, k ? st.ts[1] : st.ts[0], t & 31);
        const int ps = __shfl_sync(0xffffffffu, k ? st.ps[1] : st.ps[0], t & 31);
        if (threadIdx.x == 0) {
            if (ts == 0) {
                s_first = 0;
                s_count = 0;
            } else {
                s_first = cut_owner(st.total, G, ps);
                s_count = cut_owner(st.total, G, ps + ts - 1) - s_first + 1;
            }
        }
    }
    __syncthreads();
    float* orow = out + t * out_ts + h * out_hs;
    if (s_count == 0) {
        if (threadIdx.x < 128) orow[blockIdx.y * 128 + threadIdx.x] = 0.0f;
        return;
    }
    const size_t ss = static_cast<size_t>(H) * (R + 4);
    // a token's window spans a few CTAs' records: a shallow batch keeps registers (and occupancy)
    merge_head<R, 4>(part + static_cast<size_t>(s_first + t) * ss + static_cast<size_t>(h) * (R + 4),
                  s_count, ss, orow, 0, s_ml);
}

}  // namespace kq

namespace {

template <class G>
cudaError_t launch_partials_geo(const KqkvLaunch& a, PFN_cuTensorMapEncodeTiled_v12000 encode,
                                cudaStream_t stream) {
    using namespace kq;
    CUtensorMap tmap;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(G::D), static_cast<cuuint64_t>(a.n_kv)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.kcache_row_bytes)};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(TK)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a.kcache),
                        dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return note(cudaErrorInvalidValue);

    static uint64_t attr_set = 0;   // one bit per device ordinal, per geometry instance
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return note(e);
    if (dev >= 64 || !((attr_set >> dev) & 1)) {
        e = cudaFuncSetAttribute(kqkv_partial_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 G::SMEM_BYTES);
        if (e != cudaSuccess) return note(e);
        if (dev < 64) attr_set |= 1ull << dev;
    }
    KqParams p;
    p.q = a.q;
    p.q_hs = a.q_head_stride;
    p.q_ts = a.q_token_stride;
    p.mask = a.mask;
    p.kq_scale = a.kq_scale;
    p.n_rows = static_cast<int>(a.n_kv);
    p.part = a.part;
    p.flags = a.flags;
    p.seq_base = a.seq_base;
    p.seq_len = a.seq_len;
    p.n_seq = a.n_seq;
    return launch(kqkv_partial_kernel<G>, dim3(a.splits), dim3(NTHREADS), G::SMEM_BYTES, stream,
                  a.flags, tmap, p);
}

}  // namespace

cudaError_t launch_kqkv_partials(const KqkvLaunch& a, cudaStream_t stream) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult qres;
        void* fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                         cudaEnableDefault, &qres);
        if (e != cudaSuccess || qres != cudaDriverEntryPointSuccess || fn == nullptr)
            return note(e != cudaSuccess ? e : cudaErrorNotSupported);
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    if (a.latent == kq::GeoMistral::R) return launch_partials_geo<kq::GeoMistral>(a, encode, stream);
    if (a.latent == kq::GeoBase::R) return launch_partials_geo<kq::GeoBase>(a, encode, stream);
    return note(cudaErrorInvalidValue);
}

cudaError_t launch_kqkv_combine(const float* part, int S, int latent, float* out, int64_t out_hs,
                                uint32_t flags, cudaStream_t stream) {
    const size_t smem = 2 * static_cast<size_t>(S) * sizeof(float);
    if (smem > 48 * 1024) return note(cudaErrorInvalidValue);   // > 6144 records: not a config
    if (latent == 256)
        return launch(kq::kqkv_combine_kernel<256>, dim3(kHeads, 2), dim3(kq::CMB_THREADS), smem,
                      stream, flags, part, S, out, out_hs, 0);
    return launch(kq::kqkv_combine_kernel<kLatent>, dim3(kHeads, kLatent / 128),
                  dim3(kq::CMB_THREADS), smem, stream, flags, part, S, out, out_hs, 0);
}

cudaError_t launch_kqkv_combine_wvb(const float* part, int S, const void* w_uv, float* attn_out,
                                    int64_t attn_hs, float* out, int64_t out_hs, uint32_t flags,
                                    cudaStream_t stream) {
    const size_t smem = 2 * static_cast<size_t>(S) * sizeof(float);
    if (smem > 48 * 1024) return note(cudaErrorInvalidValue);
    return launch(kq::kqkv_combine_wvb_kernel<kLatent>, dim3(kHeads, kLatent / 128),
                  dim3(kq::CMB_THREADS), smem, stream, flags, part, S,
                  static_cast<const __half*>(w_uv), attn_out, attn_hs, out, out_hs,
                  (flags & M4B_FLAG_EARLY_RELEASE) ? 1 : 0);
}

cudaError_t launch_kqkv_ragged_combine(const float* part, const int32_t* seq_base,
                                       const int32_t* seq_len, int n_seq, int64_t n_rows,
                                       int splits, int latent, float* out, int64_t out_hs,
                                       int64_t out_ts, uint32_t flags, cudaStream_t stream) {
    if (latent == 256)
        return launch(kq::kqkv_ragged_combine_kernel<256>, dim3(kHeads, 2, n_seq),
                      dim3(kq::CMB_THREADS), 0, stream, flags, part, seq_base, seq_len, n_seq,
                      static_cast<int>(n_rows), splits, out, out_hs, out_ts);
    return launch(kq::kqkv_ragged_combine_kernel<kLatent>, dim3(kHeads, kLatent / 128, n_seq),
                  dim3(kq::CMB_THREADS), 0, stream, flags, part, seq_base, seq_len, n_seq,
                  static_cast<int>(n_rows), splits, out, out_hs, out_ts);
}

cudaError_t launch_kqkv_merge_records(const float* part, int S, int latent, float* out_records,
                                      uint32_t flags, cudaStream_t stream) {
    const size_t smem = 2 * static_cast<size_t>(S) * sizeof(float);
    if (smem > 48 * 1024) return note(cudaErrorInvalidValue);
    if (latent == 256)
        return launch(kq::kqkv_combine_kernel<256>, dim3(kHeads, 2), dim3(kq::CMB_THREADS), smem,
                      stream, flags, part, S, out_records, static_cast<int64_t>(256 + 4), 1);
    return launch(kq::kqkv_combine_kernel<kLatent>, dim3(kHeads, kLatent / 128),
                  dim3(kq::CMB_THREADS), smem, stream, flags, part, S, out_records,
                  static_cast<int64_t>(kPartStride), 1);
}

}  // namespace m4b
