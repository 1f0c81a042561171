// ovf_noalloc.cu — decode attention for callers that cannot allocate device
// memory.
//
// ovf_attention_decode needs a scratch buffer for the per-split softmax
// partials and a few counters, which the caller allocates.  Some callers
// cannot: a host whose device memory is owned by a single sanctioned
// allocator (a managed runtime or plugin host that hands out only the
// tensors it tracks), or code that must not call cudaMalloc on its hot
// path.  ovf_attention_decode_noalloc keeps that scratch in one file-scope
// device array instead, sized for the largest head layout it accepts.
//
// Contract: every GPU that loads the library holds the array (1 MiB + 1 KiB)
// until the process exits; all calls on a device share it and it keeps the
// last call's contents, so calls whose kernels overlap on the GPU (two
// streams, or two host threads) race with each other.  The array's address
// is looked up once per device, on that device's first call (see below), so
// make the first call before any stream capture begins.
#include <mutex>

#include "ovf_internal.cuh"

namespace ovf {

static constexpr size_t kNoAllocPartialBytes = 1u << 20;   // softmax partials
static constexpr size_t kNoAllocCounterInts = 256;          // one per KV head

// In host code this name is only a stand-in for the device symbol, never a
// device address: the kernel gets the address from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocPartialBytes + kNoAllocCounterInts * 4];

static void *g_noalloc_addr[64] = {nullptr};
static std::mutex g_noalloc_mu;

// Once per device, with that device current; host threads making their first
// call at the same time serialize on the mutex.  The cached address belongs to
// the device's primary context: after cudaDeviceReset the library (models,
// sessions and this address alike) must not be used on that device again.
static ovf_status noalloc_scratch_address(void **out) {
    int dev = 0;
    OVF_CUDA_TRY(cudaGetDevice(&dev));
    OVF_CHECK_ARG(dev >= 0 && dev < 64, "attention (no-alloc): device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(no-alloc attention scratch)");
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return OVF_OK;
}

}  // namespace ovf

extern "C" ovf_status ovf_attention_decode_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                                   float *out, int32_t n_heads, int32_t n_kv_heads,
                                                   int32_t head_dim, int32_t max_ctx, int32_t seq_len, float scale,
                                                   void *stream) {
    using namespace ovf;
    OVF_CHECK_ARG(q && k_cache && v_cache && out, "ComputeSingleHead (no-alloc): null buffer");
    OVF_CHECK_ARG(n_heads > 0 && n_kv_heads > 0 && head_dim > 0, "ComputeSingleHead (no-alloc): bad head layout");
    OVF_CHECK_ARG(seq_len >= 1, "ComputeSingleHead (no-alloc): seq_len must be >= 1");
    const int64_t need = attn_scratch_bytes(n_heads, n_kv_heads, head_dim);
    OVF_CHECK_ARG(need <= (int64_t)kNoAllocPartialBytes,
                  "ComputeSingleHead (no-alloc): %lld scratch bytes needed, the built-in buffer holds %lld; "
                  "use ovf_attention_decode with a caller buffer",
                  (long long)need, (long long)kNoAllocPartialBytes);
    OVF_CHECK_ARG(n_kv_heads <= (int32_t)kNoAllocCounterInts, "ComputeSingleHead (no-alloc): at most %d KV heads",
                  (int)kNoAllocCounterInts);
    void *base = nullptr;
    ovf_status st = noalloc_scratch_address(&base);
    if (st) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t *counters = reinterpret_cast<int32_t *>(static_cast<unsigned char *>(base) + kNoAllocPartialBytes);
    // The counters must start at zero; the partials are fully rewritten.
    OVF_CUDA_TRY(cudaMemsetAsync(counters, 0, (size_t)n_kv_heads * sizeof(int32_t), s));
    AttnParams p{};
    p.q = q;
    p.kc = (__half *)k_cache;
    p.vc = (__half *)v_cache;
    p.out = out;
    p.partial = static_cast<float *>(base);
    p.counters = counters;
    p.H = n_heads;
    p.KVH = n_kv_heads;
    p.hd = head_dim;
    p.max_ctx = max_ctx;
    p.seq_len_host = seq_len;
    p.scale = scale;
    return launch_attention(p, s, false);
}
