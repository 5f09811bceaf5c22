// dequant.cu -- bit-exact GGUF block dequantization on the GPU.
//
// Replaces dequantize() (src/tensor.h:451) for the types on this path.  Each
// thread produces four consecutive outputs with the reference's own fp32
// expressions (formats.cuh: dq_elem, explicit round-to-nearest mul/sub), so
// the result is bit-identical to the CPU code.  Write-bound: 4 bytes out per
// element against 0.56-1.06 bytes in.
#include <cuda_runtime.h>

#include <cstdint>

#include "formats.cuh"
#include "gemv.h"
#include "swq_device.cuh"

namespace swq {

template <int T, bool VEC>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ src,
                                                      float* __restrict__ dst, int64_t nblocks) {
    using F = Fmt<T>;
    const int64_t total4 = nblocks * (F::QK / 4);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total4; i += stride) {
        const int64_t e = i * 4;
        const int64_t b = e / F::QK;
        const int k = static_cast<int>(e - b * F::QK);
        const uint8_t* blk = src + b * F::BB;
        float4 o;
        o.x = F::dq_elem(blk, k);
        o.y = F::dq_elem(blk, k + 1);
        o.z = F::dq_elem(blk, k + 2);
        o.w = F::dq_elem(blk, k + 3);
        if (VEC) {
            *reinterpret_cast<float4*>(dst + e) = o;
        } else {
            dst[e] = o.x;
            dst[e + 1] = o.y;
            dst[e + 2] = o.z;
            dst[e + 3] = o.w;
        }
    }
}

template <int T>
static cudaError_t launch_dq(const void* src, float* dst, int64_t nblocks, int num_sms, cudaStream_t s) {
    using F = Fmt<T>;
    const int64_t total4 = nblocks * (F::QK / 4);
    int64_t grid = (total4 + 255) / 256;
    const int64_t cap = static_cast<int64_t>(num_sms) * 8;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    const bool vec = (reinterpret_cast<uintptr_t>(dst) & 15u) == 0;
    if (vec)
        dequant_kernel<T, true><<<static_cast<unsigned>(grid), 256, 0, s>>>(
            static_cast<const uint8_t*>(src), dst, nblocks);
    else
        dequant_kernel<T, false><<<static_cast<unsigned>(grid), 256, 0, s>>>(
            static_cast<const uint8_t*>(src), dst, nblocks);
    return cudaGetLastError();
}

cudaError_t dequant_launch(int type, const void* src, float* dst, int64_t nblocks, int num_sms,
                           cudaStream_t s) {
    switch (type) {
        case Q4_0: return launch_dq<Q4_0>(src, dst, nblocks, num_sms, s);
        case Q8_0: return launch_dq<Q8_0>(src, dst, nblocks, num_sms, s);
        case Q2_K: return launch_dq<Q2_K>(src, dst, nblocks, num_sms, s);
        case Q3_K: return launch_dq<Q3_K>(src, dst, nblocks, num_sms, s);
        case Q4_K: return launch_dq<Q4_K>(src, dst, nblocks, num_sms, s);
        case Q5_K: return launch_dq<Q5_K>(src, dst, nblocks, num_sms, s);
        case Q6_K: return launch_dq<Q6_K>(src, dst, nblocks, num_sms, s);
        default: return cudaErrorInvalidValue;
    }
}

SWQ_DEFINE_STATUS_FETCH(dequant)

}  // namespace swq
