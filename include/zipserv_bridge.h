/*
 * ZipServ TCA-TBE C ABI (ABI version 2) for the B200 library
 * zipserv_asplos26_b200/_lib/libzipserv_b200.so.
 *
 * Drop-in for the reference bridge: every declaration below keeps the name,
 * argument order, meaning and return convention of the symbol it replaces
 * (cited per function). Plain pointers and ints only; no Torch types. The
 * Python binding (zipserv_asplos26_b200/runtime.py) and the reference's
 * ctypes binding (integrations/vllm/zipserv_vllm/runtime.py:33-65) both bind
 * exactly these symbols.
 *
 * Conventions shared by the GPU entry points:
 *   - All device buffers belong to the caller and must stay alive until the
 *     enqueued work completes. Work is enqueued on `stream` (a cudaStream_t,
 *     NULL = legacy default stream) without host synchronisation, so calls
 *     can be captured in CUDA graphs. The only device allocation is the
 *     GEMM's K-range scratch: zipserv_mm, zipserv_mm_fp32 and
 *     zipserv_mm_kparts keep one library-owned buffer per (device, stream),
 *     allocated on the first launch that needs it (sized for every shape of the
 *     default schedule, also under stream capture) and never freed; zipserv_mm_ws
 *     takes the scratch from the caller instead.
 *   - Return 0 (cudaSuccess) or a cudaError_t value; on failure
 *     zipserv_error() describes it. Contract violations, including null
 *     pointers and device buffers not aligned to 16 bytes, return
 *     cudaErrorInvalidValue (1). N == 0 returns 0 without launching.
 *   - Shapes and pointers are validated, packed contents are not.
 */
#ifndef ZIPSERV_B200_BRIDGE_H
#define ZIPSERV_B200_BRIDGE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZIPSERV_ABI_VERSION 2

/* integrations/vllm/native/host_bridge.h:9-13. Seven independently malloc'd
 * buffers in the order sm, rare, bitmap1, bitmap2, bitmap3, medium, global;
 * lengths in bytes. Owned by the descriptor until zipserv_free(). */
typedef struct Packed {
    void* buffers[7];
    uint64_t lengths[7];
    int32_t m, k, max_common, max_rare, start_exp;
} Packed;

/* host_bridge.cpp:12. Thread-local description of the last failure. */
const char* zipserv_error(void);

/* host_bridge.cpp:13. Returns ZIPSERV_ABI_VERSION. */
int zipserv_abi_version(void);

/* host_bridge.cpp:14-16. Frees all seven buffers and nulls the pointers. */
void zipserv_free(Packed* out);

/* host_bridge.cpp:18-43. Packs a row-major BF16 m x k host matrix (m, k
 * positive multiples of 64, m*k <= INT_MAX - 4096) with the most populated
 * 7-exponent window; start_exp = uint8(base - 1). Returns 0, or -1 with the
 * descriptor zeroed and nothing allocated. Synchronous; the input must stay
 * unchanged during the call. Output is byte-identical to the reference. */
int zipserv_compress(const void* weights, int m, int k, Packed* out);

/* bridge.cu:8-21 (BF16TripleBitmap_MM_API). y[n, m] = sum_k W[m, k] x[n, k]
 * with W decoded bit-exactly from the seven buffers, FP32 accumulation and
 * BF16 output; x is [n, k] and y is [n, m], both row-major BF16.
 * split_k keeps the reference's contract (>= 1, divides k/64, workspace of
 * split_k*n*m BF16 elements required when split_k > 1) but the reduction over
 * K runs inside the kernel in FP32: the workspace is validated and never
 * written, and the kernel chooses its own K partition for the GPU. */
int zipserv_mm(void* stream, const void* sm, const void* rare, const void* b1,
               const void* b2, const void* b3, const void* medium, const void* global,
               int max_common, int max_rare, int start_exp, const void* x, void* y,
               int m, int n, int k, void* workspace, int split_k);

/* bridge.cu:23-34 (BF16TripleBitmap_Decompress_API). Writes the dense
 * row-major BF16 m x k weight, bit-exact. */
int zipserv_decode(void* stream, const void* sm, const void* rare, const void* b1,
                   const void* b2, const void* b3, const void* medium, const void* global,
                   int max_common, int max_rare, int start_exp, void* output, int m, int k);

/* bridge.cu:38-51 (BF16TripleBitmap_MM_API_FP32). Same as zipserv_mm with an
 * FP32 workspace contract (split_k*n*m floats when split_k > 1); again the
 * reduction stays in the kernel and the workspace is not written. */
int zipserv_mm_fp32(void* stream, const void* sm, const void* rare, const void* b1,
                    const void* b2, const void* b3, const void* medium, const void* global,
                    int max_common, int max_rare, int start_exp, const void* x, void* y,
                    int m, int n, int k, void* workspace, int split_k);

/* ---- Extensions (no counterpart in the reference bridge) ---------------- */

/* zipserv_mm with an explicit K partition: k_parts CTAs per 128-row block
 * (1..16, at most k/64) instead of the default persistent grid of one CTA
 * per SM. Rows whose K range is split over CTAs are summed in FP32, in K
 * order (deterministic), by the last CTA to finish them.
 * k_parts = 0 is the default schedule, as zipserv_mm uses. */
int zipserv_mm_kparts(void* stream, const void* sm, const void* rare, const void* b1,
                      const void* b2, const void* b3, const void* medium, const void* global,
                      int max_common, int max_rare, int start_exp, const void* x, void* y,
                      int m, int n, int k, int k_parts);

/* Scratch zipserv_mm_ws needs for this shape and k_parts (as in
 * zipserv_mm_kparts) on the current device: *partial_bytes for FP32 partial
 * tiles and *counter_bytes for arrival counters; both 0 when no CTA's K
 * range splits a row block. Returns 0, or cudaErrorInvalidValue (both sizes
 * 0) for an invalid shape or k_parts. */
int zipserv_mm_workspace_size(int m, int n, int k, int k_parts, uint64_t* partial_bytes,
                              uint64_t* counter_bytes);

/* zipserv_mm_kparts with caller-owned scratch; allocates nothing. Both
 * buffers 16-byte aligned and at least the sizes zipserv_mm_workspace_size
 * reports. `partials` may hold anything. `counters` must be zero-filled
 * before its first use; every launch returns the counters it used to zero,
 * so one pair of buffers (sized for the largest shape) serves any sequence
 * of launches, as long as no two of them run at the same time. Both may be
 * null when the sizes are 0. After zipserv_device_flags reports bit 0 (a
 * launch gave up on a wait), zero the counters again before the next call. */
int zipserv_mm_ws(void* stream, const void* sm, const void* rare, const void* b1,
                  const void* b2, const void* b3, const void* medium, const void* global,
                  int max_common, int max_rare, int start_exp, const void* x, void* y, int m,
                  int n, int k, int k_parts, void* partials, uint64_t partial_bytes,
                  void* counters, uint64_t counter_bytes);

/* No counterpart in the reference. zipserv_mm_kparts for callers that cannot
 * allocate device memory (bindings that hold only the buffers handed to them,
 * engines whose memory budget is fully committed at start-up): its K-range
 * scratch is a fixed 16 MiB array in the library's device memory, present on
 * every GPU that loads the library until the process exits, so the call
 * allocates nothing. Shapes needing more scratch than it holds return
 * cudaErrorInvalidValue with the sizes in zipserv_error() (the default
 * schedule fits up to 96 tokens on a 148-SM B200). The first call on a device
 * looks up the array's device address; make it before any stream capture.
 * Every call shares the one array: calls that can overlap on the GPU (other
 * streams, other threads) race and must be ordered by the caller. */
int zipserv_mm_noalloc(void* stream, const void* sm, const void* rare, const void* b1,
                       const void* b2, const void* b3, const void* medium, const void* global,
                       int max_common, int max_rare, int start_exp, const void* x, void* y,
                       int m, int n, int k, int k_parts);

/* The K partition zipserv_mm picks for this shape on the current device, or
 * a negative value if the shape is invalid. */
int zipserv_mm_plan(int m, int n, int k);

/* No counterpart in the reference. Sets how long (nanoseconds) the CTA that
 * holds the first K part of a split row block waits for the other parts'
 * FP32 pieces before it publishes its own part instead and leaves the sum to
 * the last part to arrive (default 50000; that happens when the other CTAs
 * could not start, e.g. other work holds SMs). Both ways sum in the same K
 * order, so outputs are identical; 0 makes every split row block take the
 * last-arrival route (tests use it). Applies to later launches; returns the
 * previous value. */
uint64_t zipserv_mm_reducer_wait(uint64_t ns);

/* No counterpart in the reference (its encoder runs on the host only,
 * csrc/HostPacker.h:95-183): TCA-TBE packing of a BF16 matrix that is already
 * in device memory, byte-identical to zipserv_compress. Two calls, because the
 * stream lengths depend on the data:
 *   1. zipserv_pack_device_plan: `weights` (row-major m x k BF16, 16-byte
 *      aligned), base = -1 for the most populated 7-exponent window (or a
 *      fixed window start in [0, 249]); writes the (tiles + 1) offset pairs
 *      to `global` (device, 16-byte aligned) and uses `scratch` (device,
 *      zipserv_pack_device_scratch_bytes(), 16-byte aligned). Synchronises
 *      `stream` and returns in info[0..4]: start_exp, max_common, max_rare and
 *      the byte lengths of the sm and rare streams.
 *   2. zipserv_pack_device_encode: writes sm, rare, the three bitmap planes
 *      and medium (device buffers of the lengths zipserv_compress documents)
 *      from the same weights, global and scratch, enqueued on `stream`.
 * Allocates nothing. Returns 0 or a cudaError_t (invalid arguments:
 * cudaErrorInvalidValue with zipserv_error() set). */
uint64_t zipserv_pack_device_scratch_bytes(void);
int zipserv_pack_device_plan(void* stream, const void* weights, int m, int k, int base,
                             void* global, void* scratch, int32_t* info);
int zipserv_pack_device_encode(void* stream, const void* weights, int m, int k,
                               const void* global, const void* scratch, void* sm, void* rare,
                               void* b1, void* b2, void* b3, void* medium);

/* No counterpart in the reference (row-parallel layers leave their
 * all-reduce to vLLM/NCCL): the fused GEMM of a row-parallel shard with the
 * all-reduce of its output across `world` GPUs (2..8) in the same kernel.
 * Each rank passes its K shard of W and x; every rank receives the full
 * y = sum over ranks. When a CTA holds the final FP32 value of a 32-row x
 * bn-column piece it stores it into every rank's receive buffer (peer
 * stores over NVLink; every value is one 64-bit word tagged with the launch
 * number, so no fence or flag is needed), then waits (bounded) until every
 * rank's values of its pieces carry this launch's tag, sums them in rank
 * order (so every rank stores identical BF16 outputs) and stores y.
 * recv[r] / flags[r] are rank r's receive buffer and flag area (reserved:
 * 16 bytes, unused by this version) as this process maps them (its own at
 * index rank; the others opened through zipserv_ipc_open), each at least
 * the sizes zipserv_mm_allreduce_sizes reports and zero-filled before first
 * use; `state` is this rank's 16-byte, zero-filled launch counter, advanced
 * by the kernel (so CUDA graphs may capture the call). Every rank must make
 * the same sequence of calls with the same shapes; a rank that does not
 * arrive makes the others give up after about 2 s (device flag bit 0).
 * No TMA or bulk copy reads another GPU's memory. */
int zipserv_mm_allreduce_sizes(int m, int n, int world, uint64_t* recv_bytes,
                               uint64_t* flag_bytes);
int zipserv_mm_allreduce(void* stream, const void* sm, const void* rare, const void* b1,
                         const void* b2, const void* b3, const void* medium, const void* global,
                         int max_common, int max_rare, int start_exp, const void* x, void* y,
                         int m, int n, int k, int world, int rank, void* const* recv,
                         void* const* flags, void* state, uint64_t recv_bytes,
                         uint64_t flag_bytes);
/* Device memory shared between ranks through CUDA IPC: zipserv_ipc_alloc
 * returns zero-filled memory, zipserv_ipc_handle writes its 64-byte handle,
 * zipserv_ipc_open maps another process's handle (peer access enabled),
 * zipserv_ipc_close / zipserv_ipc_free release them. */
int zipserv_ipc_alloc(uint64_t bytes, void** ptr);
int zipserv_ipc_free(void* ptr);
int zipserv_ipc_handle(void* ptr, void* handle);
int zipserv_ipc_open(const void* handle, void** ptr);
int zipserv_ipc_close(void* ptr);

/* Device-side failure flags of the current device (bit 0: a pipeline wait
 * in a kernel gave up after its iteration limit; results of that launch are
 * undefined). Reading synchronises the device; clear != 0 resets the flags.
 * Returns a cudaError_t. */
int zipserv_device_flags(unsigned* flags, int clear);

#ifdef __cplusplus
}
#endif
#endif
