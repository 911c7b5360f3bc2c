// tp_allreduce.cu — one-shot all-reduce (fp32 sum) over NVLink peer memory
// for the tensor-parallel decode step.
//
// At decode sizes the residual all-reduce is a few KB to a few hundred KB,
// where a collective library's protocol overhead is most of its cost. Each
// rank here owns a receive buffer with one slot per source rank, mapped into
// every peer through CUDA IPC. The kernel writes this rank's vector straight
// into its slot on every peer (plain stores over NVLink), raises one flag per
// (source rank, slice) on every peer, waits for the peers' flags in its own
// memory, then sums the slots in rank order, so every rank ends with the same
// bits. Two buffer generations alternate, so a rank that runs ahead writes
// into the generation its peers finished reading. With a handoff
// (ForgeArHandoff, int4, up to 4 sequences) the slices are whole 128-groups
// and each summed group is also staged for the RMSNorm GEMV that reads x
// next: the codes of gain * x in that GEMV's input-block layout, and the
// group's sum of squares of x.
//
// Every wait is bounded (%globaltimer; 2 s, or FORGE_WAIT_NS at set-up): on
// expiry the kernel sets the handle's error word and returns.
#include <cstdlib>
#include <cstring>
#include <vector>
#include "common.cuh"
#include "forge_internal.h"
#include "gemv_core.cuh"
#include "../../include/forge_b200.h"

namespace {
constexpr int kSlices = 16;      // CTAs per all-reduce; each owns a contiguous slice
constexpr int kThreads = 256;
constexpr int kMaxRanks = 8;

struct ArDev {
    float* peer_buf[kMaxRanks];     // rank r's receive buffer [2][T][cap]
    uint32_t* peer_flag[kMaxRanks]; // rank r's flags [2][T][kSlices]
    uint32_t* epoch;                // this rank's [kSlices] counters
    int T, rank, cap;
    unsigned long long wait_ns;     // limit of each flag wait (FORGE_WAIT_NS at set-up)
};

// Flag-wait limit: FORGE_WAIT_NS from the environment (nanoseconds, at least
// 1 ms), else the library's 2 s.
unsigned long long wait_limit_ns() {
    const char* e = getenv("FORGE_WAIT_NS");
    const unsigned long long v = e ? strtoull(e, nullptr, 10) : 0ull;
    return v >= 1000000ull ? v : (unsigned long long)FORGE_WAIT_NS;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kThreads) k_tp_allreduce(float* x, int n, const ArDev d, uint32_t* err,
                                                           const ForgeArHandoff ho) {
    __shared__ uint32_t s_ep;
    __shared__ int s_ok;
    const int sl = blockIdx.x;
    int s0, s1;
    if (ho.pq) {  // slices of whole 128-groups (the handoff quantises groups)
        const int gps = ((n >> 7) + kSlices - 1) / kSlices;
        s0 = min(n, sl * gps * 128);
        s1 = min(n, (sl + 1) * gps * 128);
    } else {
        const int per = ((n + kSlices - 1) / kSlices + 3) & ~3;  // whole float4s per slice
        s0 = sl * per;
        s1 = min(n, s0 + per);
    }
    // Under programmatic dependent launch the next kernel (the next GEMV)
    // may start now and stream its weights while this exchange runs; this
    // kernel itself waits for the one that wrote x. The epoch counters are
    // this kernel's own (the previous all-reduce took its value at its start,
    // and uses the other buffer generation).
    pdl_trigger();
    if (threadIdx.x == 0) {
        s_ep = d.epoch[sl] + 1;
        d.epoch[sl] = s_ep;
        s_ok = 1;
    }
    pdl_wait();
    __syncthreads();
    const uint32_t ep = s_ep;
    const int gen = ep & 1;
    const size_t slot = ((size_t)gen * d.T + d.rank) * d.cap;
    // 1. this rank's slice into its slot on every rank (peer stores over NVLink)
    for (int r = 0; r < d.T; ++r) {
        float* dst = d.peer_buf[r] + slot;
        for (int i = s0 + 4 * (int)threadIdx.x; i < s1; i += 4 * kThreads) {
            if (i + 4 <= s1) {
                *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(x + i);
            } else {
                for (int k = i; k < s1; ++k) dst[k] = x[k];
            }
        }
    }
    __syncthreads();
    // 2. flags: "slice sl of rank `rank`, generation ep, has landed" (the
    // release orders the CTA's data stores, made visible by the barrier,
    // before the flag)
    if (threadIdx.x < d.T)
        st_release_sys(d.peer_flag[threadIdx.x] + ((size_t)gen * d.T + d.rank) * kSlices + sl, ep);
    // 3. wait for every rank's flag of this slice in this rank's memory
    if (threadIdx.x < d.T) {
        const volatile uint32_t* f = d.peer_flag[d.rank] + ((size_t)gen * d.T + threadIdx.x) * kSlices + sl;
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (*f != ep) {
            if ((++spins & 1023u) == 0 && globaltimer_ns() - t0 > d.wait_ns) {
                atomicOr(err, FORGE_DEVERR_COUNTER_TIMEOUT);
                s_ok = 0;
                break;
            }
        }
        (void)ld_acquire_sys(const_cast<const uint32_t*>(f));  // orders the data reads after the flag
    }
    __syncthreads();
    if (!s_ok) return;
    // 4. sum the slots in rank order (the same bits on every rank)
    const float* base = d.peer_buf[d.rank] + (size_t)gen * d.T * d.cap;
    if (!ho.pq) {
        for (int i = s0 + (int)threadIdx.x; i < s1; i += kThreads) {
            float acc = base[i];
            for (int r = 1; r < d.T; ++r) acc += __ldcv(base + (size_t)r * d.cap + i);
            x[i] = acc;
        }
        return;
    }
    // 5. with the handoff, one warp per 128-group: the sum, then the next
    // GEMV's input staged from it — the codes of gain * x (int8 hi/lo,
    // scale, column sums) and the group's sum of squares of x, from which
    // that GEMV forms its RMSNorm factor
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, G = ho.d >> 7;
    for (int gs = s0 + 128 * warp; gs < s1; gs += 128 * (kThreads / 32)) {
        const int i = gs + 4 * lane;
        float4 acc = *reinterpret_cast<const float4*>(base + i);
        for (int r = 1; r < d.T; ++r) {
            const float4 v = __ldcv(reinterpret_cast<const float4*>(base + (size_t)r * d.cap + i));
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        *reinterpret_cast<float4*>(x + i) = acc;
        const int b = gs / ho.d, kk = gs - b * ho.d;
        const float4 gv = __ldg(reinterpret_cast<const float4*>(ho.gain + kk + 4 * lane));
        float ss = acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) ho.ssq[b * G + (kk >> 7)] = ss;
        pq_group_warp(make_float4(gv.x * acc.x, gv.y * acc.y, gv.z * acc.z, gv.w * acc.w), kk >> 7, b,
                      2 * ho.batch, G, ho.pq);
    }
}
}  // namespace

struct ForgeTpAr {
    ArDev dev{};
    void* local = nullptr;   // receive buffers + flags (one allocation, mapped by every peer)
    uint32_t* epoch = nullptr;
    ForgeTpFusedDev fused{};          // host copy
    ForgeTpFusedDev* fused_dev = nullptr;
    uint32_t* tile_epoch = nullptr;
    std::vector<void*> opened;
};

// Allocates this rank's receive buffer (capacity `cap` floats per source
// rank) and maps every peer's through CUDA IPC, exchanging the handles over
// the NCCL communicator. All ranks call it together.
int forge_tp_ar_init(void* comm, int rank, int T, int cap, cudaStream_t stream, ForgeTpAr** out) {
    if (T < 2 || T > kMaxRanks || cap <= 0) return forge_fail(-1, "tp all-reduce: %d ranks (2..%d)", T, kMaxRanks);
    ForgeTpAr* ar = new ForgeTpAr();
    cap = (cap + 15) & ~15;
    const int max_tiles = cap / 16;  // 16-row tiles of a vector of cap rows
    const size_t buf_bytes = (size_t)2 * T * cap * 4, flag_bytes = (size_t)2 * T * kSlices * 4;
    // the GEMV epilogue exchange has its own buffers and per-tile flags
    const size_t fbuf_off = buf_bytes + flag_bytes, fbuf_bytes = (size_t)2 * T * cap * 4;
    const size_t fflag_off = fbuf_off + fbuf_bytes, fflag_bytes = (size_t)2 * T * max_tiles * 4;
    const size_t total = fflag_off + fflag_bytes;
    if (cudaMalloc(&ar->local, total) != cudaSuccess || cudaMemset(ar->local, 0, total) != cudaSuccess ||
        cudaMalloc(&ar->epoch, kSlices * 4) != cudaSuccess || cudaMemset(ar->epoch, 0, kSlices * 4) != cudaSuccess ||
        cudaMalloc(&ar->tile_epoch, (size_t)max_tiles * 4) != cudaSuccess ||
        cudaMemset(ar->tile_epoch, 0, (size_t)max_tiles * 4) != cudaSuccess ||
        cudaMalloc(&ar->fused_dev, sizeof(ForgeTpFusedDev)) != cudaSuccess) {
        cudaGetLastError();
        forge_tp_ar_destroy(ar);
        return forge_fail(-1, "tp all-reduce: device allocation failed");
    }
    cudaIpcMemHandle_t mine;
    if (cudaIpcGetMemHandle(&mine, ar->local) != cudaSuccess) {
        cudaGetLastError();
        forge_tp_ar_destroy(ar);
        return forge_fail(-1, "tp all-reduce: cudaIpcGetMemHandle failed");
    }
    // all-gather the 64-byte handles through device memory
    const size_t hb = sizeof(cudaIpcMemHandle_t);
    void* dh = nullptr;
    std::vector<char> all(hb * T);
    int rc = 0;
    if (cudaMalloc(&dh, hb * (T + 1)) != cudaSuccess) rc = forge_fail(-1, "tp all-reduce: handle buffer");
    if (!rc && cudaMemcpy((char*)dh + hb * T, &mine, hb, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = forge_fail(-1, "tp all-reduce: handle upload");
    if (!rc) rc = forge_tp_allgather_f32(comm, (const float*)((char*)dh + hb * T), (float*)dh, hb / 4, stream);
    if (!rc && (cudaStreamSynchronize(stream) != cudaSuccess ||
                cudaMemcpy(all.data(), dh, hb * T, cudaMemcpyDeviceToHost) != cudaSuccess))
        rc = forge_fail(-1, "tp all-reduce: handle exchange");
    if (dh) cudaFree(dh);
    for (int r = 0; r < T && !rc; ++r) {
        void* p = ar->local;
        if (r != rank) {
            cudaIpcMemHandle_t h;
            memcpy(&h, all.data() + hb * r, hb);
            if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                rc = forge_fail(-1, "tp all-reduce: cudaIpcOpenMemHandle of rank %d failed", r);
                break;
            }
            ar->opened.push_back(p);
        }
        ar->dev.peer_buf[r] = (float*)p;
        ar->dev.peer_flag[r] = (uint32_t*)((char*)p + buf_bytes);
        ar->fused.buf[r] = (float*)((char*)p + fbuf_off);
        ar->fused.flag[r] = (uint32_t*)((char*)p + fflag_off);
    }
    if (rc) {
        forge_tp_ar_destroy(ar);
        return rc;
    }
    ar->dev.epoch = ar->epoch;
    ar->dev.T = T;
    ar->dev.rank = rank;
    ar->dev.cap = cap;
    ar->dev.wait_ns = wait_limit_ns();
    ar->fused.tile_epoch = ar->tile_epoch;
    ar->fused.T = T;
    ar->fused.rank = rank;
    ar->fused.cap = cap;
    ar->fused.max_tiles = max_tiles;
    if (cudaMemcpy(ar->fused_dev, &ar->fused, sizeof(ForgeTpFusedDev), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        forge_tp_ar_destroy(ar);
        return forge_fail(-1, "tp all-reduce: exchange descriptor upload");
    }
    *out = ar;
    return 0;
}

const ForgeTpFusedDev* forge_tp_fused_dev(const ForgeTpAr* ar) { return ar ? ar->fused_dev : nullptr; }

void forge_tp_ar_destroy(ForgeTpAr* ar) {
    if (!ar) return;
    for (void* p : ar->opened) cudaIpcCloseMemHandle(p);
    if (ar->local) cudaFree(ar->local);
    if (ar->epoch) cudaFree(ar->epoch);
    if (ar->tile_epoch) cudaFree(ar->tile_epoch);
    if (ar->fused_dev) cudaFree(ar->fused_dev);
    delete ar;
}

int forge_tp_ar_capacity(const ForgeTpAr* ar) { return ar ? ar->dev.cap : 0; }

int forge_tp_ar_sum_f32(ForgeTpAr* ar, float* x, int n, uint32_t* err, cudaStream_t stream, const ForgeArHandoff* handoff) {
    if (!ar || n <= 0 || n > ar->dev.cap) return forge_fail(-1, "tp all-reduce: %d floats above capacity", n);
    ForgeArHandoff ho{};
    if (handoff && handoff->pq) {
        if (handoff->d % 128 || n != handoff->batch * handoff->d || handoff->batch > 4 || !handoff->ssq || !handoff->gain)
            return forge_fail(-1, "tp all-reduce: bad handoff shape");
        ho = *handoff;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kSlices);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_tp_allreduce, x, n, (const ArDev)ar->dev, err, (const ForgeArHandoff)ho) != cudaSuccess)
        return forge_fail(-1, "tp all-reduce launch: %s", cudaGetErrorString(cudaGetLastError()));
    return forge_check_launch("tp all-reduce");
}

// Self-test of the bounded peer wait, on one GPU, with no peer: the
// exchange buffers of T ranks all live in this process's memory and only
// rank 0 runs its all-reduce, so its waits for the flags of ranks 1..T-1
// (which nothing raises) run out after wait_ns. Reports the device error
// bits and the kernel's wall time, then checks that the context still runs
// work (a second, one-rank launch that needs no flags). 0 when the launch
// ended and the context is usable; the error bits say whether it timed out.
extern "C" FORGE_API int forge_tp_selftest_absent_peer(int T, int n, unsigned long long wait_ns, uint32_t* err_bits,
                                                       double* ms) {
    if (T < 2 || T > kMaxRanks || n <= 0 || n > (1 << 20) || wait_ns < 1000000ull || !err_bits || !ms)
        return forge_fail(FORGE_INVALID_ARGS, "forge_tp_selftest_absent_peer: bad args");
    const int cap = (n + 15) & ~15;
    const size_t buf_bytes = (size_t)2 * T * cap * 4, flag_bytes = (size_t)2 * T * kSlices * 4;
    void* local = nullptr;
    uint32_t *epoch = nullptr, *err = nullptr;
    float* x = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    if (cudaMalloc(&local, buf_bytes + flag_bytes) != cudaSuccess || cudaMemset(local, 0, buf_bytes + flag_bytes) ||
        cudaMalloc(&epoch, kSlices * 4) != cudaSuccess || cudaMemset(epoch, 0, kSlices * 4) ||
        cudaMalloc(&err, 16) != cudaSuccess || cudaMemset(err, 0, 16) || cudaMalloc(&x, 4 * (size_t)n) != cudaSuccess ||
        cudaMemset(x, 0, 4 * (size_t)n) || cudaEventCreate(&e0) || cudaEventCreate(&e1))
        rc = forge_fail(-1, "forge_tp_selftest_absent_peer: device allocation failed");
    if (!rc) {
        ArDev d{};
        for (int r = 0; r < T; ++r) {  // every "peer" is this process's own buffer
            d.peer_buf[r] = (float*)local;
            d.peer_flag[r] = (uint32_t*)((char*)local + buf_bytes);
        }
        d.epoch = epoch;
        d.T = T;
        d.rank = 0;
        d.cap = cap;
        d.wait_ns = wait_ns;
        cudaEventRecord(e0);
        k_tp_allreduce<<<kSlices, kThreads>>>(x, n, d, err, ForgeArHandoff{});
        cudaEventRecord(e1);
        if (cudaEventSynchronize(e1) != cudaSuccess) {
            rc = forge_fail(-1, "forge_tp_selftest_absent_peer: %s", cudaGetErrorString(cudaGetLastError()));
        } else {
            float t = 0.f;
            cudaEventElapsedTime(&t, e0, e1);
            *ms = t;
            cudaMemcpy(err_bits, err, 4, cudaMemcpyDeviceToHost);
            // the context still runs work: one rank alone needs no flags
            d.T = 1;
            cudaMemset(err, 0, 4);
            k_tp_allreduce<<<kSlices, kThreads>>>(x, n, d, err, ForgeArHandoff{});
            uint32_t e2 = 0;
            if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(&e2, err, 4, cudaMemcpyDeviceToHost) != cudaSuccess ||
                e2 != 0)
                rc = forge_fail(-1, "forge_tp_selftest_absent_peer: context unusable after the timeout");
        }
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    for (void* p : {local, (void*)epoch, (void*)err, (void*)x})
        if (p) cudaFree(p);
    return rc;
}
