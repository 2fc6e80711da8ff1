// zipserv_mm_noalloc: the fused GEMM for callers that cannot allocate device
// memory. Some callers have no allocator of their own to reach (a Go or Java
// binding that holds only the buffers handed to it), and some are not allowed
// to allocate once they are running (a serving engine that gave its whole
// memory budget to a pre-sized pool at start-up, or code that must not call
// cudaMalloc in its hot path). The fused GEMM needs scratch whenever a row
// block's K range is split across CTAs (FP32 partial tiles plus arrival
// counters). zipserv_mm and friends allocate it on first use, and
// zipserv_mm_ws needs the caller to provide it. This entry point instead
// uses a fixed array in the library's own device memory, which the driver
// places when the library's device code is loaded on a GPU and keeps there
// until the process exits.
//
// Included by zipserv_cuda.cu after capi_cuda.cu (it uses mm_impl).
#include <mutex>

namespace {

// The scratch, one copy per GPU that loads the library: arrival counters in
// the first kNoAllocCounterBytes, FP32 partial tiles after them. 16 MiB
// covers the default schedule up to 96 tokens on a 148-SM B200 (partial tiles
// take 148 CTAs x 2 x (N tile / 4) x 2 KB) for any M and K.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr size_t kNoAllocCounterBytes = size_t(256) << 10;
constexpr size_t kNoAllocPartialBytes = kNoAllocScratchBytes - kNoAllocCounterBytes;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// In host code g_noalloc_scratch names a host-side stand-in, not device
// memory: the device address of each GPU's copy is looked up once per device
// (with that device current) and kept here.
unsigned char* g_noalloc_base[zs::kMaxDevices] = {};
std::mutex g_noalloc_mutex;

cudaError_t noalloc_base(int device, unsigned char** base) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_base[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            char msg[160];
            snprintf(msg, sizeof(msg), "zipserv_mm_noalloc: scratch address lookup failed: %s",
                     cudaGetErrorString(e));
            zs_set_error(msg);
            return e;
        }
        g_noalloc_base[device] = static_cast<unsigned char*>(p);
    }
    *base = g_noalloc_base[device];
    return cudaSuccess;
}

}  // namespace

extern "C" int zipserv_mm_noalloc(void* stream, const void* sm, const void* rare, const void* b1,
                                  const void* b2, const void* b3, const void* medium,
                                  const void* global, int max_common, int max_rare,
                                  int start_exp, const void* x, void* y, int m, int n, int k,
                                  int k_parts) {
    if (k_parts < 0 || k_parts > 16 || (zs::valid_matrix(m, k) && k_parts > k / 64)) {
        zs_set_error("k_parts must be in [0, min(16, K/64)]");
        return int(cudaErrorInvalidValue);
    }
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Every request goes through the caller-scratch path, so the library's
    // own allocating workspace is never reached; invalid shapes and n == 0
    // return from mm_impl before any scratch is used.
    zs::GemmScratch scratch{nullptr, 0, nullptr, 0};
    if (zs::valid_gemm(m, n, k, 1) && n > 0) {
        int device = 0;
        cudaError_t e = cudaGetDevice(&device);
        if (e != cudaSuccess) return int(e);
        if (device < 0 || device >= zs::kMaxDevices) return int(cudaErrorInvalidDevice);
        size_t need_p = 0, need_c = 0;
        zs::gemm_workspace_bytes(m, n, k, k_parts, device, &need_p, &need_c);
        if (need_p > kNoAllocPartialBytes || need_c > kNoAllocCounterBytes) {
            char msg[240];
            snprintf(msg, sizeof(msg),
                     "zipserv_mm_noalloc: this shape needs %zu bytes of partial tiles and %zu of "
                     "counters; the fixed scratch holds %zu and %zu (use zipserv_mm or "
                     "zipserv_mm_ws for it)",
                     need_p, need_c, kNoAllocPartialBytes, kNoAllocCounterBytes);
            zs_set_error(msg);
            return int(cudaErrorInvalidValue);
        }
        unsigned char* base = nullptr;
        if ((e = noalloc_base(device, &base)) != cudaSuccess) return int(e);
        // The array keeps whatever the previous call left; the counters must
        // start at zero (a launch that gave up on a wait may not have reset
        // them), the partial tiles may hold anything.
        if (need_c && (e = cudaMemsetAsync(base, 0, need_c, s)) != cudaSuccess) return int(e);
        scratch = zs::GemmScratch{base + kNoAllocCounterBytes, kNoAllocPartialBytes, base,
                                  kNoAllocCounterBytes};
    }
    return int(mm_impl(s, sm, rare, b1, b2, b3, medium, global, max_common, max_rare,
                       start_exp & 255, x, y, m, n, k, nullptr, 1, k_parts, &scratch));
}
