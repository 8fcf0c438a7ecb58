// fg_attention_noalloc.cu -- tree attention for callers that cannot allocate.
//
// fg_tree_attention takes its split-K scratch from the caller.  Some callers
// have no way to provide it: a trainer or runtime that binds this C ABI from
// another language with no handle on a device allocator, or a host framework
// whose memory manager owns the whole GPU, where calling cudaMalloc would
// either fail or synchronize the device in the middle of a rollout round.
// fg_tree_attention_noalloc serves them from one fixed buffer that lives in
// the library itself: a file-scope __device__ array of FG_NOALLOC_SCRATCH_BYTES
// that every GPU which loads the library keeps until the process exits.
//
// Rules for callers:
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * All calls share the one buffer, so calls that overlap on the GPU (two
//    streams, or two host threads on one device) race; serialize them.
//  * A call whose scratch need exceeds FG_NOALLOC_SCRATCH_BYTES is rejected
//    with FG_ECAPACITY (ask fewer splits, or use fg_tree_attention).
//  * A bf16 call that splits the KV range clears the split counters with a
//    cudaMemsetAsync on the stream first (the previous call may have used the
//    array with another layout), so unlike fg_tree_attention it does not start
//    early under the kernel before it (programmatic dependent launch).  fp32
//    calls use no scratch at all.
//  * The device address is cached per device ordinal; after cudaDeviceReset
//    the cached address is stale, so a process that resets a device must not
//    call this entry point on it again.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include <atomic>

#include "fg_common.cuh"

// The shared scratch.  In host code this name is only a host-side stand-in
// for the device array; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_fg_noalloc_scratch[FG_NOALLOC_SCRATCH_BYTES];

namespace fg {

// Per-device address cache.  Host threads may race on a device's first call:
// each then looks the address up itself and stores the same value, and the
// atomics make those reads and writes well defined.
static void* noalloc_scratch_ptr() {
    static std::atomic<void*> ptrs[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    void* p = ptrs[dev].load(std::memory_order_acquire);
    if (p == nullptr) {
        const cudaError_t e = cudaGetSymbolAddress(&p, g_fg_noalloc_scratch);
        if (e != cudaSuccess) {
            set_cuda_error(e);
            return nullptr;
        }
        ptrs[dev].store(p, std::memory_order_release);
    }
    return p;
}

}  // namespace fg

extern "C" fg_status fg_tree_attention_noalloc(const void* q, int32_t dtype, const fg_kv_layer* kv,
                                               const int32_t* kv_len, const uint32_t* anc_bits, int32_t B,
                                               int32_t n_nodes, int32_t n_q_heads, int32_t n_kv_heads,
                                               int32_t head_dim, float scale, void* out, int32_t num_splits,
                                               int32_t max_kv_len, void* stream) {
    if (B == 0) return FG_OK;
    if (!kv || B < 0 || n_nodes <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads) return FG_EINVAL;
    const int32_t kv_max = max_kv_len > 0 ? max_kv_len : kv->capacity;
    if (dtype == FG_DTYPE_F32)  // the fp32 kernel keeps no split-K partials
        return fg_tree_attention(q, dtype, kv, kv_len, anc_bits, B, n_nodes, n_q_heads, n_kv_heads, head_dim, scale,
                                 out, nullptr, 0, num_splits, kv_max, stream);
    const size_t need = fg_tree_attention_workspace_size(B, n_nodes, n_q_heads, n_kv_heads, head_dim, num_splits,
                                                         kv_max);
    if (need > (size_t)FG_NOALLOC_SCRATCH_BYTES) return FG_ECAPACITY;
    void* scratch = nullptr;
    if (need > 0) {
        scratch = fg::noalloc_scratch_ptr();
        if (!scratch) return FG_ECUDA;
        // the split counters (the last plan.items int32 of the layout, one per
        // row group of a KV head) must start at zero
        const size_t items =
            (size_t)plan_attention(B, n_nodes, n_q_heads, n_kv_heads, num_splits, kv_max).items;
        const cudaError_t e = cudaMemsetAsync(static_cast<uint8_t*>(scratch) + need - items * sizeof(int32_t), 0,
                                              items * sizeof(int32_t), (cudaStream_t)stream);
        if (e != cudaSuccess) {
            fg::set_cuda_error(e);
            return FG_ECUDA;
        }
    }
    return fg_tree_attention(q, dtype, kv, kv_len, anc_bits, B, n_nodes, n_q_heads, n_kv_heads, head_dim, scale, out,
                             scratch, need, num_splits, kv_max, stream);
}
