/*
 * m4b.h -- C ABI of the B200 (sm_100a) implementation of aubier's fused MLA decode-attention ops.
 *
 * The reference (jmars/aubier) exposes the path as three ggml custom ops, dispatched by the
 * patched ggml-cuda backend (patches/ggml-m4/custom-op-m4.patch, ggml-cuda.cu:2504-2512):
 *
 *   GGML_OP_M4_WKB    ggml_cuda_m4_wkb(ctx, dst)    patches/ggml-m4/m4-wkb.cu:71-86
 *   GGML_OP_M4_KQKV   ggml_cuda_m4_kqkv(ctx, dst)   patches/ggml-m4/m4-kqkv.cu:340-378
 *   GGML_OP_M4_PHASE  ggml_cuda_m4_phase(ctx, dst)  patches/ggml-m4/m4-phase.cu:205-277
 *
 * Each entry point below replaces the body of one of those launchers: a ggml-cuda shim copies
 * dst->src[i] (data, type, ne[], nb[]), dst and dst->op_params into the POD argument struct and
 * calls the entry point on ctx.stream(); a nonzero return becomes GGML_ABORT, the reference's
 * assert-on-contract behaviour.  Plain pointers and sizes only: no ggml, torch or CUDA types.
 *
 * Contract shared by every launch entry point (the reference's, patches/README.md:16-18):
 *   - one stream, plain kernel launches, no host synchronisation and no allocation, so a call is
 *     legal inside CUDA-graph capture; scratch memory is passed in by the caller;
 *   - device pointers only; a host pointer is a caller bug (the reference's ops have no CPU path:
 *     ggml-cpu.c:2064-2082 aborts);
 *   - shapes, types and strides are validated before any launch; a violation returns
 *     M4B_EINVAL and launches nothing (the reference's GGML_ASSERTs, e.g. m4-kqkv.cu:345-355).
 *
 * Geometries (engine/m1_layer.h:47-55 and the BASELINE shape; selected from the tensors' shapes,
 * never from a flag):
 *   BASELINE      32 heads, q_nope 128, rope 64, latent 512, K row 576, V head 128, f16 W_UK/W_UV
 *   MISTRAL_SMALL 32 heads, q_nope 64,  rope 64, latent 256, K row 320, V head 128, Q8_0 W_UK/W_UV
 *
 * Tensor layouts use ggml conventions: ne[0] is the innermost (contiguous) dimension, nb[] are
 * byte strides, types are ggml_type ids.
 */
#ifndef M4B_H
#define M4B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define M4B_ABI_VERSION 1

#if defined(__GNUC__)
#define M4B_API __attribute__((visibility("default")))
#else
#define M4B_API
#endif

/* The stream argument is a cudaStream_t (NULL = legacy default stream). */
typedef struct CUstream_st * m4b_stream_t;

/* Return codes. */
enum m4b_status {
    M4B_OK       = 0,
    M4B_EINVAL   = 1, /* shape / type / stride / alignment contract violated: nothing launched */
    M4B_ESCRATCH = 2, /* scratch missing or smaller than the m4b_*_scratch_bytes() requirement */
    M4B_ECUDA    = 3, /* a CUDA runtime call or launch failed */
    M4B_EDEVICE  = 4, /* the current device is not an sm_100 part */
    M4B_ENOTSUP  = 5, /* valid ggml op, but a geometry / phase this build does not implement */
    M4B_ETIMEOUT = 6  /* reported by m4b_device_status(): a kernel's bounded wait gave up */
};

/* ggml_type ids (vendor/llama.cpp/ggml/include/ggml.h) of the types these ops accept. */
enum m4b_type {
    M4B_TYPE_F32  = 0,
    M4B_TYPE_F16  = 1,
    M4B_TYPE_Q8_0 = 8,
    M4B_TYPE_I32  = 26,
    M4B_TYPE_I64  = 27
};

/* One operand: the fields of ggml_tensor the kernels read. */
typedef struct m4b_tensor {
    void *   data;   /* device pointer; NULL marks an absent optional operand */
    int32_t  type;   /* enum m4b_type */
    int32_t  _pad;
    int64_t  ne[4];  /* elements per dimension, ne[0] innermost */
    uint64_t nb[4];  /* byte strides */
} m4b_tensor;

/* Launch flags (all optional). */
enum m4b_flags {
    /* launch with programmatic stream serialisation: the kernel may start while the previous
       kernel on the stream drains and waits (griddepcontrol.wait) before touching its inputs */
    M4B_FLAG_PDL       = 1u << 0,
    /* with M4B_FLAG_PDL: the KV cache is not written by the kernels immediately before this one,
       so KQKV may start streaming it before the preceding kernel finishes */
    M4B_FLAG_KV_STATIC = 1u << 1,
    /* m4b_wkb only (additive): also copy each query head's rope half -- the 64 floats that follow
       q_nope in src1's head row -- into dst's head row right after the latent, so dst holds the
       graph's Qcur = concat(q_abs, q_pe) (engine/m1_layer.cpp:443-447) without a separate copy.
       Needs src1's head stride >= nope + 64 floats and dst's >= latent + 64 floats. */
    M4B_FLAG_QCAT      = 1u << 2,
    /* with M4B_FLAG_PDL on PHASE selector 2 and m4b_exchange_merge_wvb: release the next kernel
       of the stream as soon as this one's W_UV loads are issued, instead of at completion, so the
       next layer's weight loads overlap this merge.  The next kernel still waits for this one's
       results.  Measured, one-GPU layer-steps on the same box: 16.9 -> 16.0 us at 4,096 keys,
       23.4 -> 22.0 at 32,768, 46.0 -> 45.2 at 131,072, and +0.7 % layer-steps/s at 262,144 keys.
       Other entry points ignore it. */
    M4B_FLAG_EARLY_RELEASE = 1u << 3
};

/*
 * GGML_OP_M4_WKB -- the MLA absorption gemv, q_abs[h] = W_UK[h] . q_nope[h].
 * Replaces ggml_cuda_m4_wkb (patches/ggml-m4/m4-wkb.cu:71-86); builder ggml_m4_wkb
 * (vendor/llama.cpp/ggml/src/ggml.c:3398-3423).
 *   src0  W_UK    F16 [128, 512, 32]  (BASELINE)   |  Q8_0 [64, 256, 32]  (MISTRAL_SMALL)
 *   src1  q_nope  F32 [128, 32, T]    any head stride nb[1] (the engine's view has 768 / 512 B)
 *   dst   q_abs   F32 [512, 32, T]    any head stride nb[1] >= 4*ne[0] (may point into Qcur)
 * T = 1 in the reference's op.  Additively, 1 <= T <= 64 tokens (token stride nb[2]) share one
 * read of W_UK: the ragged batch path (m4b_kqkv_ragged).
 */
typedef struct m4b_wkb_args {
    m4b_tensor src0, src1, dst;
    uint32_t   flags;
} m4b_wkb_args;

M4B_API int m4b_wkb(const m4b_wkb_args * args, m4b_stream_t stream);

/*
 * GGML_OP_M4_KQKV -- fused scores + masked softmax + V contraction over the shared latent KV cache.
 * Replaces ggml_cuda_m4_kqkv (patches/ggml-m4/m4-kqkv.cu:340-378); builder ggml_m4_kqkv
 * (ggml.c:3425-3459).  op_params[0] = kq_scale.
 *   src0  kcache  F16 [576, N, 1, 1]   N >= 1 dynamic; nb[1] multiple of 16; V = rows [0, 512)
 *   src1  q       F32 [576, 32, 1, 1]  head stride nb[1]
 *   src2  mask    F32 [N, 1, 1, 1]     0 / -INF (optional here: data == NULL means all zero)
 *   dst   out     F32 [512, 1, 32, 1]  head stride nb[2]; a fully masked head yields 0
 * Needs scratch >= m4b_kqkv_scratch_bytes(geometry, N) (split-K partials; the reference keeps
 * them in a static device array, m4-kqkv.cu:52-72).
 */
typedef struct m4b_kqkv_args {
    m4b_tensor src0, src1, src2, dst;
    float      kq_scale;
    uint32_t   flags;
    void *     scratch;
    uint64_t   scratch_bytes;
} m4b_kqkv_args;

M4B_API int m4b_kqkv(const m4b_kqkv_args * args, m4b_stream_t stream);

/*
 * KQKV, split-K partials only (no reference counterpart: the additive op the multi-GPU and fused
 * paths use; the partial is the (m, l, o) record of m4-kqkv.cu:306-311).
 *   dst  partials F32 [516, 32, S, 1] contiguous: per (split, head) o[512] then m (log2 units),
 *        l, 2 pad floats.  1 <= S <= min(m4b_kqkv_max_splits(), ceil(N / 128)); split s
 *        covers a balanced contiguous run of 128-key tiles.
 * src0..src2 and kq_scale as for m4b_kqkv; scratch unused.
 */
M4B_API int m4b_kqkv_partials(const m4b_kqkv_args * args, m4b_stream_t stream);

/*
 * KQKV over a ragged batch (no reference counterpart: the reference runs its fused ops only at one
 * token per step, m1_layer.cpp:283-297, and falls back to stock ops for batches).  Token t
 * attends to its own window of one packed cache -- rows [seq_base[t], seq_base[t] + seq_len[t]),
 * the engine's per-row mask (m1_layer.cpp:756-773) -- with the single-token op's numerics.
 *   kcache    F16 [576, R, 1, 1]  as src0 of m4b_kqkv (all tokens' windows, in any order)
 *   q         F32 [576, 32, T]    per-token query: head stride nb[1], token stride nb[2]
 *   seq_base  I32 [T]             device memory, never read on the host (it may be produced on
 *   seq_len   I32 [T]             the device); a window outside [0, R) counts as empty and makes
 *                                 m4b_device_status() report M4B_EINVAL
 *   dst       F32 [512, T, 32]    token stride nb[1], head stride nb[2]; an empty window gives 0
 * 1 <= T <= 64.  The tiles of all windows are spread evenly over the SMs, whatever the lengths.
 * Needs scratch >= m4b_kqkv_ragged_scratch_bytes(T).  With M4B_FLAG_KV_STATIC the windows, like
 * the cache, must not be written by the kernels immediately before this one.
 */
typedef struct m4b_kqkv_ragged_args {
    m4b_tensor kcache, q, seq_base, seq_len, dst;
    float      kq_scale;
    uint32_t   flags;
    void *     scratch;
    uint64_t   scratch_bytes;
} m4b_kqkv_ragged_args;

M4B_API int m4b_kqkv_ragged(const m4b_kqkv_ragged_args * args, m4b_stream_t stream);
M4B_API uint64_t m4b_kqkv_ragged_scratch_bytes(int64_t n_tokens);

/*
 * KQKV for callers that cannot allocate (no counterpart in the reference, whose KQKV always uses
 * its own static array; here the regular entry point takes caller scratch instead).  Same
 * operands, contract and output as m4b_kqkv; args->scratch is ignored.  The split-K partial
 * records live in a fixed device array inside the library (148 splits x 32 heads x 2064 B =
 * 9.8 MB per GPU, held until exit); a call needing more records returns M4B_ESCRATCH.  The first
 * call on a device looks the array's address up (cudaGetSymbolAddress) with that device current:
 * make it before any stream capture.  Calls on one device share the array: calls whose kernels
 * overlap on the GPU race.  Allocates nothing (no cudaMalloc / cudaFree).
 */
M4B_API int m4b_kqkv_static_scratch(const m4b_kqkv_args * args, m4b_stream_t stream);

/*
 * GGML_OP_M4_PHASE -- the remaining per-token phases, selected by op_params[0].
 * Replaces ggml_cuda_m4_phase (patches/ggml-m4/m4-phase.cu:205-277); builders
 * ggml_m4_phase_kvwrite / ggml_m4_phase_wvb (ggml.c:3461-3539).
 *   phase 0  KV-write   (MISTRAL_SMALL geometry, the reference's selector 0, m4-phase.cu:97-200):
 *                       src0 cur F32 [4096]; src1 W_kva Q8_0 [4096, 320]; src2 kv norm weight
 *                       F32 [256]; src3 kcache F16 [320, N] (written in place at row kidx[0]);
 *                       src4 kidx I64 [1]; src5 pos I32 [1] (both read on the device only);
 *                       dst Kcur F32 [320].  Kcur and the norm weight 8-byte aligned, cache
 *                       rows 4-byte aligned.  A row outside the cache writes nothing and makes
 *                       m4b_device_status() report M4B_EINVAL.  BASELINE has no W_kva: M4B_ENOTSUP
 *   phase 1  WVB        src0 W_UV F16 [512, 128, 32]; src1 x F32 [512, T, 32] (nb[2] head
 *                       stride); dst F32 [128, T, 32].  T = 1 in the reference's op; additively
 *                       1 <= T <= 64 tokens (token stride nb[1]) share one read of W_UV
 *   phase 2  COMBINE_WVB (additive selector): src0 W_UV F16 [512, 128, 32]; src1 partials
 *                       F32 [516, 32, S] (m4b_kqkv_partials layout, 1 <= S <= 6144, e.g.
 *                       gathered from several GPUs); dst F32 [128, 1, 32]; optional src2 F32
 *                       [512, 1, 32] receives the merged attention output.  Needs scratch
 *                       >= m4b_phase_scratch_bytes(2) unless src2 is given.
 *   phase 3  MERGE      (additive selector): src1 partial records F32 [516, 32, S]; dst F32
 *                       [516, 32, 1]: one unnormalised record per head (o = sum a_s o_s,
 *                       m = max m_s, l = sum a_s l_s, a_s = 2^(m_s - m)) -- what one GPU sends to
 *                       the others in the KV-slab exchange; phase 2 merges the gathered records.
 * op_params follow ggml.c:3464-3468 (an int32 array): [0] phase, [1..6] rope f32, [7] eps,
 * [8] n_dims, [9] n_ctx_orig.
 */
typedef struct m4b_phase_args {
    m4b_tensor src[6];
    m4b_tensor dst;
    int32_t    op_params[16];
    uint32_t   flags;
    void *     scratch;
    uint64_t   scratch_bytes;
} m4b_phase_args;

M4B_API int m4b_phase(const m4b_phase_args * args, m4b_stream_t stream);

/*
 * KV-append into a sharded cache (additive; the reference keeps the whole cache on one GPU,
 * engine/m1_engine.cpp:2165): PHASE selector 0 (args as m4b_phase, op_params[0] = 0) for a cache
 * split into contiguous slabs of rows, one per GPU.  kidx[0] is the new row's index in the WHOLE
 * cache; src[3] is this GPU's slab, which holds rows [slab_base, slab_base + src[3].ne[1]).  Every
 * GPU computes Kcur (dst); only the GPU whose slab holds the row writes it.  A row held by another
 * slab is skipped without error; a negative kidx sets M4B_EINVAL in m4b_device_status, as
 * selector 0 does for a row outside its cache.  slab_base < 0 is refused (M4B_EINVAL).
 */
M4B_API int m4b_phase_kvwrite_slab(const m4b_phase_args * args, int64_t slab_base,
                                   m4b_stream_t stream);

/*
 * The KV-slab exchange between the GPUs of one node, fused into the merge kernels (no counterpart
 * in the reference, which runs on one GPU: engine/m1_engine.cpp:2165).  One process per GPU; each
 * GPU computes split-K records over its slab of the cache (m4b_kqkv_partials), then
 *   m4b_exchange_publish     merges them into one record per head and stores that record into
 *                            every peer's receive buffer over NVLink (CUDA IPC mappings), each
 *                            value tagged with the exchange's epoch; src[1] = records [516, 32, S]
 *   m4b_exchange_combine_wvb waits (bounded) until every GPU's record of the current exchange has
 *                            arrived, merges them and applies W_UV, in one kernel: src[0] = W_UV,
 *                            dst = F32 [128, 1, 32]; the optional src[2] (F32 [512, 1, 32])
 *                            receives the merged attention.  No scratch.
 * Set-up (not capture-safe, once per process): m4b_exchange_create allocates this GPU's buffer;
 * exchange the M4B_IPC_HANDLE_BYTES handles of all ranks (m4b_exchange_ipc_handle) through any
 * host channel, then m4b_exchange_open with all of them, rank-ordered.  The two launch entry
 * points are plain launches (capturable); every GPU must call them the same number of times.
 * A peer that never publishes makes the combine give up after the wait limit (~1 s by default,
 * m4b_set_wait_limit_cycles) and report M4B_ETIMEOUT through m4b_device_status(); the output of
 * that call is undefined.
 * Tear-down: every rank calls m4b_exchange_detach (unmaps the peers' buffers), then all ranks meet
 * on the host, then each calls m4b_exchange_destroy (frees its own buffer) -- an exporting process
 * must not free a buffer that another process still has mapped.
 */
#define M4B_IPC_HANDLE_BYTES 64
typedef struct m4b_exchange m4b_exchange;

M4B_API int m4b_exchange_create(int world, int rank, m4b_exchange ** out);
M4B_API int m4b_exchange_ipc_handle(const m4b_exchange * x, void * handle_out);
M4B_API int m4b_exchange_open(m4b_exchange * x, const void * handles);
/* Set-up when every rank's exchange lives in this one process (one host thread or process driving
 * several GPUs, as ggml-cuda's multi-GPU backend does): all[r] is rank r's exchange, created here
 * on its own device, n == world.  The peers' buffers are used through their own pointers (peer
 * access between the devices is enabled; no IPC mapping), so tear-down needs no meeting: destroy
 * the exchanges once no launch uses them.  Kernels of different ranks that wait on each other
 * must run on different GPUs; on one GPU, run every rank's publish before any rank's combine. */
M4B_API int m4b_exchange_open_local(m4b_exchange * x, m4b_exchange * const * all, int n);
M4B_API int m4b_exchange_detach(m4b_exchange * x);
M4B_API int m4b_exchange_destroy(m4b_exchange * x);
M4B_API int m4b_exchange_publish(m4b_exchange * x, const m4b_phase_args * args, m4b_stream_t stream);
M4B_API int m4b_exchange_combine_wvb(m4b_exchange * x, const m4b_phase_args * args,
                                     m4b_stream_t stream);
/* publish + combine_wvb in one launch: src[0] W_UV, src[1] this GPU's records [516, 32, S],
 * optional src[2] attention output, dst as combine_wvb.  Every GPU calls it once per exchange. */
M4B_API int m4b_exchange_merge_wvb(m4b_exchange * x, const m4b_phase_args * args,
                                   m4b_stream_t stream);

/* Sizes.  geometry: 0 = BASELINE, 1 = MISTRAL_SMALL. */
M4B_API uint64_t m4b_kqkv_scratch_bytes(int geometry, int64_t n_kv);
M4B_API uint64_t m4b_phase_scratch_bytes(int phase);
M4B_API int      m4b_kqkv_default_splits(int64_t n_kv); /* the split count m4b_kqkv uses */
M4B_API int      m4b_kqkv_max_splits(void);

/*
 * The reference's supports_op (ggml-cuda.cu:5848-5885) for the three ops: 1 when the shapes and
 * types match a supported geometry (no launch, no CUDA call, no memory read), 0 otherwise.
 * op: 0 = WKB, 1 = KQKV, 2 = PHASE (phase from op_params[0]).  srcs: up to 6 operands, dst: the
 * output.  A NULL data marks an absent optional operand; a present operand that has no memory yet
 * (ggml asks while scheduling, before allocation) may carry any non-NULL, 256-byte-aligned
 * placeholder.  KQKV with srcs[3] / srcs[4] present (and no mask) is the ragged batch form of
 * m4b_kqkv_ragged: srcs[3] = seq_base, srcs[4] = seq_len, dst F32 [latent, T, 32].
 */
M4B_API int m4b_supports_op(int op, const m4b_tensor * srcs, int n_srcs, const m4b_tensor * dst,
                    const int32_t * op_params);

/*
 * The tri-state enable flag of the engine (LoopArgs::m4_*, engine/m1_session.h:152-166, resolved
 * in engine/m1_engine.cpp:2170-2197 and gated in engine/m1_layer.cpp:283-297):
 * flag -1 = AUTO (on iff gpu_core), 0 = off (stock ops), 1 = explicit on (needs gpu_core).
 * Writes the resolved on/off to *enabled (on also requires nt == 1 unless the op supports the
 * ragged extension) and returns M4B_OK, or M4B_EINVAL for explicit 1 without gpu_core or a flag
 * outside {-1, 0, 1}.
 */
M4B_API int m4b_resolve_flag(int flag, int gpu_core, int nt, int ragged_ok, int * enabled);

/* Reads and clears the device status word; synchronises the stream.  M4B_OK, M4B_ETIMEOUT (a
   bounded wait gave up) or M4B_EINVAL (a ragged window outside the cache). */
M4B_API int m4b_device_status(m4b_stream_t stream);

/*
 * Sets how long every bounded wait of the kernels lasts before it gives up (SM clock cycles; the
 * default, also restored by cycles <= 0, is 2^31, about 1 s).  No counterpart in the reference,
 * whose kernels never wait on another agent.  Limits below 2^20 cycles act as 2^20.  Applies to
 * the current device; synchronises it, so call it outside stream capture and with no kernel of
 * this library in flight.  A test shortens the limit to make a wait that nothing will end (an
 * exchange whose peer never publishes) run out in milliseconds.
 */
M4B_API int m4b_set_wait_limit_cycles(int64_t cycles);

/* The last CUDA runtime error (a cudaError_t value; 0 = none) behind an M4B_ECUDA from a launch
   entry point, with its name in *name when name is not NULL.  Reading clears it. */
M4B_API int m4b_last_cuda_error(const char ** name);

M4B_API const char * m4b_strerror(int code);
M4B_API int          m4b_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* M4B_H */
