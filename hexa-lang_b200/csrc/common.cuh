// common.cuh — device helpers shared by the forge_b200 kernels (sm_100a).
//
// PTX wrappers for mbarriers, 1-D bulk async copies (cp.async.bulk, no
// multicast), programmatic dependent launch, bf16 bit handling and the
// bounded waits every spin in this library goes through.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define FORGE_DEV __device__ __forceinline__

// Error flag bits written by kernels into the handle's device status word.
enum : uint32_t {
    FORGE_DEVERR_MBAR_TIMEOUT = 1u,   // an mbarrier wait ran out of iterations
    FORGE_DEVERR_COUNTER_TIMEOUT = 2u, // a flag / counter spin ran out
    FORGE_DEVERR_BAD_INDEX = 4u,       // a token id or position out of range
};

// Bounded spins: every wait gives up after FORGE_WAIT_NS of wall time (read
// from %globaltimer) or FORGE_SPIN_LIMIT polls, whichever comes first, then
// raises an error bit that the host reads. Normal waits last microseconds.
#define FORGE_WAIT_NS (2000000000ull)
#define FORGE_SPIN_LIMIT (1u << 30)

FORGE_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
FORGE_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
FORGE_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
FORGE_DEV void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
FORGE_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 ::"r"(smem_u32(bar)) : "memory");
}
FORGE_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
FORGE_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Non-blocking probe of a phase (never suspends the thread) — for a
// thread that must keep doing other work (issuing copies) while it polls.
FORGE_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity to complete. Returns false (and
// raises the device error flag) when the spin budget runs out.
FORGE_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < FORGE_SPIN_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && globaltimer_ns() - t0 > FORGE_WAIT_NS) break;
    }
    if (err) atomicOr(err, FORGE_DEVERR_MBAR_TIMEOUT);
    return false;
}

// --------------------------------------------------------- bulk async copy
// Global -> shared 1-D bulk copy completing on an mbarrier (tx bytes). Both
// addresses 16-byte aligned, size a multiple of 16. No multicast.
FORGE_DEV void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// The same copy for data a step reads once (weights, scales, cached K/V
// rows), marked evict-first in L2: the stream then does not push out of L2
// what is read again soon (activations, split partials, kernel code).
FORGE_DEV uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
FORGE_DEV void bulk_g2s_stream(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// L2 prefetch of a global range (no smem destination).
FORGE_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------- programmatic launch
// Every kernel calls pdl_wait() before touching data written by the kernel
// launched before it, and pdl_trigger() once its own CTAs may be joined by
// the next kernel's CTAs (which then stream their weights early).
FORGE_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FORGE_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ------------------------------------------------------------ named barrier
FORGE_DEV void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------- bf16 bits
FORGE_DEV float bf16_lo_f32(uint32_t v) { return __uint_as_float(v << 16); }
FORGE_DEV float bf16_hi_f32(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
FORGE_DEV uint16_t f32_to_bf16_bits(float f) {
    __nv_bfloat16 b = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&b);
}
FORGE_DEV float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Splits x into hi + lo bf16 parts (hi = RN(x), lo = RN(x - hi)); hi + lo
// carries ~16 significant bits of x, so a bf16 tensor-core product with both
// parts reproduces an fp32 activation to ~2^-17 relative.
FORGE_DEV void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    hi = f32_to_bf16_bits(x);
    lo = f32_to_bf16_bits(x - bf16_bits_to_f32(hi));
}

FORGE_DEV uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    // (a & b) | c
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// mma.sync m16n8k16 bf16 x bf16 -> fp32 (A row-major, B col-major).
FORGE_DEV void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                              const float (&c)[4]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// mma.sync m16n8k32 u8 (A, codes) x s8 (B, activations) -> s32, exact.
FORGE_DEV void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Unpacks the two words of one 16x32 int4 k-tile (layout.cuh) into the four
// u8 A-fragment registers: low nibbles are rows g, high nibbles rows g+8.
FORGE_DEV void dequant_q4_u8(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    a[0] = w0 & 0x0F0F0F0Fu;
    a[1] = (w0 >> 4) & 0x0F0F0F0Fu;
    a[2] = w1 & 0x0F0F0F0Fu;
    a[3] = (w1 >> 4) & 0x0F0F0F0Fu;
}

// Dequantises one packed int4 word (8 codes, code = q + 7) into the four
// bf16x2 A-fragment registers of a 16x16 tile. Nibble j and j+4 land in the
// low/high halves of register j; 0x4300|n is the bf16 value 128+n, and
// subtracting 135 leaves q exactly.
FORGE_DEV void dequant_q4_word(uint32_t w, uint32_t (&a)[4]) {
    const uint32_t mask = 0x000F000Fu, magic = 0x43004300u;
    const __nv_bfloat162 bias = __halves2bfloat162(__ushort_as_bfloat16((unsigned short)0x4307),
                                                   __ushort_as_bfloat16((unsigned short)0x4307));
    uint32_t r[4];
    r[0] = lop3_and_or(w, mask, magic);
    r[1] = lop3_and_or(w >> 4, mask, magic);
    r[2] = lop3_and_or(w >> 8, mask, magic);
    r[3] = lop3_and_or(w >> 12, mask, magic);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&r[i]);
        v = __hsub2(v, bias);
        a[i] = *reinterpret_cast<uint32_t*>(&v);
    }
}
