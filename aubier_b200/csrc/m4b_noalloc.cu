// m4b_noalloc.cu -- m4b_kqkv_static_scratch: GGML_OP_M4_KQKV for callers that cannot allocate.
//
// m4b_kqkv needs scratch for its split-K partial records and takes it from the caller.  Some
// callers have no allocator to take it from: code that must not call cudaMalloc at all (a plugin
// running inside a host application that owns every device allocation, a real-time loop where an
// allocation can stall or fail, or a pipeline that checks for zero allocations after start-up).
// For them this entry point runs the same two kernels with the partial records in one fixed
// device array that is part of the library image.
//
// The array is file-scope static device memory of a fixed size: every GPU that loads the library
// keeps it (kStaticRecords records, 9.8 MB) until the process exits.  Host code cannot use the
// array's name as a device address (in host code it names a host-side stand-in), so the first
// call on a device -- with that device current -- asks the runtime for the real address with
// cudaGetSymbolAddress and caches it per device; make that first call before any stream capture.
// The cache lives as long as the process's primary context on that device: after a
// cudaDeviceReset the library image, and with it the array, is loaded again, possibly elsewhere,
// so a process that resets a device must not call this entry point on it afterwards.  Concurrent
// first calls from several host threads all store the same address (the cache entries are
// atomic, so this is well defined).
// All calls on a device share the array and it keeps whatever the last call wrote: every split
// writes its whole record before the merge reads it, so nothing needs clearing, but two calls
// whose kernels overlap on the GPU (two streams, no ordering between them) race on the records.
// The call allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.
#include "m4b_internal.h"

namespace m4b {
namespace noalloc {

constexpr int kStaticRecords = kMaxSplits * kHeads;   // 148 splits x 32 heads, up to 2064 B each

static __device__ __align__(256) float g_kqkv_static_part[kStaticRecords * kPartStride];

// cached device address of the array, per device ordinal (nullptr until the first call there)
std::atomic<float*> g_addr[64] = {};

}  // namespace noalloc
}  // namespace m4b

extern "C" M4B_API int m4b_kqkv_static_scratch(const m4b_kqkv_args* a, m4b_stream_t stream) {
    using namespace m4b;
    if (!a) return M4B_EINVAL;
    int geom = 0;
    int rc = check_kqkv(*a, &geom);
    if (rc != M4B_OK) return rc;
    int sms = 0;
    rc = device_check(&sms);
    if (rc != M4B_OK) return rc;
    const int splits = default_splits(a->src0.ne[1], sms);
    if (static_cast<int64_t>(splits) * kHeads > noalloc::kStaticRecords)
        return M4B_ESCRATCH;   // more split records than the static array holds
    int dev = 0;
    if (note(cudaGetDevice(&dev)) != cudaSuccess) return M4B_ECUDA;
    if (dev < 0 || dev >= 64) return M4B_EDEVICE;
    float* part = noalloc::g_addr[dev].load(std::memory_order_acquire);
    if (part == nullptr) {
        void* p = nullptr;
        if (note(cudaGetSymbolAddress(&p, noalloc::g_kqkv_static_part)) != cudaSuccess ||
            p == nullptr)
            return M4B_ECUDA;
        part = static_cast<float*>(p);
        noalloc::g_addr[dev].store(part, std::memory_order_release);
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = launch_kqkv_partials(make_kqkv_launch(*a, geom, splits, part), s);
    if (e != cudaSuccess) return M4B_ECUDA;
    e = launch_kqkv_combine(part, splits, kGeo[geom].latent, static_cast<float*>(a->dst.data),
                            static_cast<int64_t>(a->dst.nb[2] / 4), a->flags & M4B_FLAG_PDL, s);
    return e == cudaSuccess ? M4B_OK : M4B_ECUDA;
}
