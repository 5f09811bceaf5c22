// swq_device.cuh -- device helpers shared by the libswq kernels (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace swq {

// GGMLType ids, src/gguf.h:18-40.
enum : int { Q4_0 = 2, Q8_0 = 8, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14 };

// Device-side status word: bounded waits OR a code in here and give up.
// Read and cleared by swq_check().
enum : unsigned { DEV_TIMEOUT_FULL = 1u, DEV_TIMEOUT_EMPTY = 2u, DEV_TIMEOUT_DRAIN = 4u,
                  DEV_TIMEOUT_MMA = 8u, DEV_TIMEOUT_PEER = 16u,
                  DEV_BAD_ALIGN = 32u,    // not a wait: an input the kernel skipped
                  DEV_BAD_ID = 64u };     // not a wait: an expert id out of range
// One word per translation unit (no relocatable device code); each unit
// exports a host accessor through SWQ_DEFINE_STATUS_FETCH.
static __device__ unsigned g_swq_dev_status = 0;

#define SWQ_DEFINE_STATUS_FETCH(name)                                              \
    cudaError_t status_fetch_##name(unsigned* out, cudaStream_t s) {                \
        unsigned zero = 0;                                                          \
        cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_swq_dev_status, sizeof(unsigned), \
                                                  0, cudaMemcpyDeviceToHost, s);    \
        if (e != cudaSuccess) return e;                                             \
        e = cudaStreamSynchronize(s);                                               \
        if (e != cudaSuccess) return e;                                             \
        if (*out == 0) return cudaSuccess;                                          \
        e = cudaMemcpyToSymbolAsync(g_swq_dev_status, &zero, sizeof(unsigned), 0,  \
                                    cudaMemcpyHostToDevice, s);                     \
        if (e != cudaSuccess) return e;                                             \
        return cudaStreamSynchronize(s);                                            \
    }

// Upper bound for every spin-wait, in nanoseconds of %globaltimer (~0.5 s).
constexpr uint64_t kWaitLimitNs = 500ull * 1000ull * 1000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, for at most kWaitLimitNs.
// Returns false on timeout (and records `code` in the device status word).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_swq_dev_status, code);
            return false;
        }
    }
}

// ---- bulk async copy (TMA, non-tensor) ----------------------------------------

// global -> shared, completes `bytes` of transaction on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.  Destination: this CTA only.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar, uint64_t l2_policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(l2_policy)
        : "memory");
}

// Weights are streamed once per call: evict-first keeps them from pushing the
// activations and outputs out of L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---- programmatic dependent launch -------------------------------------------

__device__ __forceinline__ void pdl_wait_primary() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- named barriers -----------------------------------------------------------

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- fp16 -> fp32 --------------------------------------------------------------

// IEEE half bits -> float bits, the same mapping as the reference's
// fp16_to_fp32 (src/tensor.h:33-58): subnormals renormalised, Inf/NaN keep
// their payload.  Integer-only so that NaN payloads survive bit-exactly.
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            // Leading one of the 10-bit mantissa at bit p; shift it to bit 10.
            const int p = 31 - __clz(mant);
            const int sh = 10 - p;
            mant = (mant << sh) & 0x3FFu;
            bits = sign | (static_cast<uint32_t>(113 - sh) << 23) | (mant << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (mant << 13);
    }
    return __uint_as_float(bits);
}

// ---- small integer helpers ----------------------------------------------------

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// 32-bit little-endian load from shared memory at a 2-byte aligned address.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
    return static_cast<uint32_t>(q[0]) | (static_cast<uint32_t>(q[1]) << 16);
}

__device__ __forceinline__ uint32_t lds_u32_a4(const uint8_t* p) {
    return *reinterpret_cast<const uint32_t*>(p);
}

// Four consecutive little-endian words at a 2-byte aligned shared-memory
// address: five aligned 32-bit loads and funnel shifts (by 0 or 16 bits)
// instead of eight 16-bit loads.  Reads up to 4 bytes past the region.
__device__ __forceinline__ void lds_u32x4_a2(const uint8_t* p, uint32_t (&w)[4]) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 2u) << 3;
    uint32_t v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = base[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

__device__ __forceinline__ uint4 lds_u128(const uint8_t* p) {
    return *reinterpret_cast<const uint4*>(p);
}

}  // namespace swq
