// tp.cu — tensor-parallel plumbing: NCCL loaded at run time, and the shard
// plan shared by every rank.
//
// NCCL is opened with dlopen ("libnccl.so.2", or the file FORGE_NCCL_LIB
// names) the first time a tensor-parallel handle needs it, so the library
// loads on machines without NCCL and single-GPU use never touches it. The
// collectives are the two of the Megatron decode split: an fp32 sum of the
// residual stream after the row-split O and down projections, and a max over
// the packed 64-bit argmax keys of the vocabulary-split LM head (the
// reference's NCCL call site for the all-reduce: hxccl_linux_emit.hexa:493).
#include <dlfcn.h>
#include <mutex>
#include <nccl.h>
#include "forge_internal.h"
#include "../../include/forge_b200.h"

namespace {
struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*comm_destroy)(ncclComm_t);
    const char* (*error_string)(ncclResult_t);
};

Nccl* nccl() {
    static Nccl api{};
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* path = getenv("FORGE_NCCL_LIB");
        void* lib = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return;
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(lib, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(lib, "ncclCommInitRank");
        api.all_reduce = (decltype(api.all_reduce))dlsym(lib, "ncclAllReduce");
        api.all_gather = (decltype(api.all_gather))dlsym(lib, "ncclAllGather");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(lib, "ncclCommDestroy");
        api.error_string = (decltype(api.error_string))dlsym(lib, "ncclGetErrorString");
        ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.all_gather && api.comm_destroy &&
             api.error_string;
    });
    return ok ? &api : nullptr;
}

int nccl_fail(const char* what, ncclResult_t r) {
    Nccl* n = nccl();
    return forge_fail(-1, "%s: %s", what, n ? n->error_string(r) : "NCCL unavailable");
}
}  // namespace

int forge_tp_comm_init(void** comm, const void* unique_id, int rank, int size) {
    Nccl* n = nccl();
    if (!n) return forge_fail(-1, "tensor parallel: libnccl.so.2 could not be loaded (set FORGE_NCCL_LIB)");
    ncclUniqueId id;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    memcpy(&id, unique_id, sizeof(id));
    ncclComm_t c = nullptr;
    ncclResult_t r = n->comm_init_rank(&c, size, id, rank);
    if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
    *comm = c;
    return 0;
}

void forge_tp_comm_destroy(void* comm) {
    if (Nccl* n = nccl())
        if (comm) n->comm_destroy((ncclComm_t)comm);
}

int forge_tp_allreduce_sum_f32(void* comm, float* buf, size_t count, cudaStream_t stream) {
    ncclResult_t r = nccl()->all_reduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)comm, stream);
    return r == ncclSuccess ? 0 : nccl_fail("ncclAllReduce(sum)", r);
}

int forge_tp_allreduce_max_u64(void* comm, unsigned long long* buf, size_t count, cudaStream_t stream) {
    ncclResult_t r = nccl()->all_reduce(buf, buf, count, ncclUint64, ncclMax, (ncclComm_t)comm, stream);
    return r == ncclSuccess ? 0 : nccl_fail("ncclAllReduce(max)", r);
}

int forge_tp_allgather_f32(void* comm, const float* send, float* recv, size_t count, cudaStream_t stream) {
    ncclResult_t r = nccl()->all_gather(send, recv, count, ncclFloat32, (ncclComm_t)comm, stream);
    return r == ncclSuccess ? 0 : nccl_fail("ncclAllGather", r);
}

extern "C" {
// Contiguous split of n items in units of `gran` over `size` ranks: the first
// (n/gran) % size ranks take one unit more. Ranks that get nothing are an
// error (the caller's shard would be empty).
FORGE_API int forge_tp_split(int64_t n, int64_t gran, int rank, int size, int64_t* off, int64_t* len) {
    if (!off || !len || n <= 0 || gran <= 0 || size <= 0 || rank < 0 || rank >= size || n % gran)
        return forge_fail(FORGE_INVALID_ARGS, "forge_tp_split: bad args");
    const int64_t units = n / gran, base = units / size, extra = units % size;
    const int64_t mine = base + (rank < extra ? 1 : 0);
    if (mine == 0) return forge_fail(FORGE_INVALID_ARGS, "forge_tp_split: %lld units over %d ranks leaves rank %d empty",
                                     (long long)units, size, rank);
    *off = (rank * base + (rank < extra ? rank : extra)) * gran;
    *len = mine * gran;
    return 0;
}

FORGE_API int forge_b200_tp_unique_id(void* out) {
    if (!out) return forge_fail(FORGE_INVALID_ARGS, "forge_b200_tp_unique_id: null buffer");
    Nccl* n = nccl();
    if (!n) return forge_fail(-1, "forge_b200_tp_unique_id: libnccl.so.2 could not be loaded (set FORGE_NCCL_LIB)");
    ncclUniqueId id;
    ncclResult_t r = n->get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    memcpy(out, &id, sizeof(id));
    return 0;
}
}  // extern "C"
