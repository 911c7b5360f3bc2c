// noalloc.cu — split-K flash-decode for callers that cannot allocate device
// memory.
//
// forge_flash_decode needs a caller-provided workspace (split partials and
// merge counters). Some callers have no way to provide one: a host runtime
// whose device memory is owned entirely by another allocator (for example a
// farr mirror table that only hands out existing buffers), code running
// while a stream is being captured into a CUDA graph, or a deployment with a
// fixed device-memory budget that must not grow after start-up. This file
// gives them an entry that allocates nothing: its scratch lives in one
// file-scope __device__ array of FORGE_FD_NOALLOC_SCRATCH_BYTES bytes, which
// every GPU that loads the library holds until the process exits.
//
// All calls on a device share that array, and it keeps whatever the last
// call left in it, so two calls that overlap on the GPU (different streams,
// or different threads without ordering) race and corrupt each other's
// results; order them on one stream. Each call clears the merge counters it
// uses before its kernel runs, so a call never depends on the previous
// call's contents.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (host code cannot use the symbol itself: in host code
// it names a host-side stand-in, not device memory). That lookup is done
// once per device, with the device current; make the first call on each
// device before any stream capture begins. The address is kept for the life
// of the process, so the entry must not be used after cudaDeviceReset (or
// any other teardown of the device's primary context): the kept address
// would name memory of a context that no longer exists.
//
// Errors found by the kernel (a position outside the cache, a wait that ran
// out) are recorded in a device word of this file, separate from the
// library's other error words; forge_flash_decode_noalloc_status reads and
// clears it. No other entry of the library uses this array or this word.
#include <mutex>
#include "forge_internal.h"
#include "../../include/forge_b200.h"

#ifndef FORGE_FD_NOALLOC_SCRATCH_BYTES
#define FORGE_FD_NOALLOC_SCRATCH_BYTES (4ll << 20)  // 4 MiB per device
#endif

namespace {
constexpr int64_t kScratchBytes = FORGE_FD_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_fd_scratch[kScratchBytes];

void* g_scratch_ptr[64] = {nullptr};
uint32_t* g_err_ptr[64] = {nullptr};
static __device__ uint32_t g_fd_err;
std::mutex g_mu;

// Device address of the scratch array (and of the error word) on the
// current device; looked up once per device.
int scratch_for_device(void** scratch, uint32_t** err) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_decode_noalloc: no current CUDA device");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_fd_scratch);
        if (e != cudaSuccess || !p)
            return forge_fail(-1, "forge_flash_decode_noalloc: cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        void* q = nullptr;
        e = cudaGetSymbolAddress(&q, g_fd_err);
        if (e != cudaSuccess || !q)
            return forge_fail(-1, "forge_flash_decode_noalloc: cudaGetSymbolAddress(error word): %s", cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
        g_err_ptr[dev] = (uint32_t*)q;
    }
    *scratch = g_scratch_ptr[dev];
    *err = g_err_ptr[dev];
    return 0;
}
}  // namespace

extern "C" {
FORGE_API int64_t forge_flash_decode_noalloc_capacity(void) { return kScratchBytes; }

FORGE_API int forge_flash_decode_noalloc(const float* q, const uint16_t* kc, const uint16_t* vc,
                                         const int32_t* pos, int B, int H, int Hkv, int hd, int lmax,
                                         float* out, void* stream) {
    if (!q || !kc || !vc || !pos || !out || B <= 0 || H <= 0 || Hkv <= 0 || lmax <= 0)
        return forge_fail(FORGE_INVALID_ARGS, "forge_flash_decode_noalloc: bad args");
    const int64_t need = forge_flash_decode_workspace_bytes(B, H, Hkv, hd, lmax);
    if (need < 0 || need > kScratchBytes)
        return forge_fail(FORGE_INVALID_ARGS,
                          "forge_flash_decode_noalloc: B=%d H=%d hd=%d lmax=%d needs %lld scratch bytes, above "
                          "the fixed %lld-byte array; use forge_flash_decode with a workspace",
                          B, H, hd, lmax, (long long)need, (long long)kScratchBytes);
    void* scratch = nullptr;
    uint32_t* err = nullptr;
    if (int rc = scratch_for_device(&scratch, &err)) return rc;
    if (forge_attn_configure()) return -1;
    ForgeAttnArgs a{};
    a.q = q; a.kc = kc; a.vc = vc; a.pos = pos; a.B = B; a.H = H; a.Hkv = Hkv; a.hd = hd; a.lmax = lmax;
    a.nsplit = forge_attn_pick_splits(B, Hkv, lmax);
    const int64_t counters = ((int64_t)B * Hkv * 4 + 255) / 256 * 256;
    a.counters = (uint32_t*)scratch;
    a.partial = (float*)((char*)scratch + counters);
    a.out = out;
    a.err = err;
    // merge tickets must start at zero whatever an earlier call left behind
    cudaError_t e = cudaMemsetAsync(scratch, 0, (size_t)B * Hkv * 4, (cudaStream_t)stream);
    if (e != cudaSuccess) return forge_fail(-1, "forge_flash_decode_noalloc: clearing counters: %s", cudaGetErrorString(e));
    return forge_attn_launch(a, (cudaStream_t)stream, false) ? FORGE_INVALID_ARGS : 0;
}

// Waits for all work on the current device (every stream, including
// non-blocking ones), then reads and clears the error word the
// allocation-free kernel writes (a position outside the cache, a wait that
// ran out).
FORGE_API int forge_flash_decode_noalloc_status(void) {
    void* scratch = nullptr;
    uint32_t* err = nullptr;
    if (int rc = scratch_for_device(&scratch, &err)) return rc;
    if (cudaError_t se = cudaDeviceSynchronize(); se != cudaSuccess)
        return forge_fail(-1, "forge_flash_decode_noalloc_status: %s", cudaGetErrorString(se));
    uint32_t e = 0;
    if (cudaMemcpyFromSymbol(&e, g_fd_err, sizeof(e)) != cudaSuccess)
        return forge_fail(-1, "forge_flash_decode_noalloc_status: %s", cudaGetErrorString(cudaGetLastError()));
    if (e) {
        const uint32_t zero = 0;
        cudaMemcpyToSymbol(g_fd_err, &zero, sizeof(zero));
        return forge_fail(-1, "forge_flash_decode_noalloc: kernel error word 0x%x", e);
    }
    return 0;
}
}  // extern "C"
