// allreduce.cu -- one-shot sum all-reduce of an fp32 vector across the GPUs of
// a tensor-parallel group, over peer memory (NVLink / NVSwitch).
//
// Tensor-parallel decode adds the partial products of the row-parallel
// projections (o and down) once per layer: a few to a few hundred KB, where a
// ring or tree all-reduce spends its time in latency.  Here every rank keeps one
// buffer that all ranks map (CUDA IPC); one launch per call does:
//
//   CTA b owns the same slice of the vector on every rank.
//   1. copy my slice into my buffer (data half e % 2 of epoch e);
//   2. publish epoch e in my flag word b (release, system scope);
//   3. wait until every peer's flag word b holds e (acquire, bounded);
//   4. read slice b of every rank's buffer and sum in rank order 0..G-1.
//
// Every rank sums the same values in the same order, so all ranks end with the
// same bits.  A slice only depends on the same CTA of the other ranks: there is
// no grid-wide barrier.  Epochs live in device memory (a per-CTA counter in
// the rank's own buffer), so a launch captured in a CUDA graph advances them on
// every replay.  Two data halves suffice: a rank cannot publish epoch e + 2
// before every peer has published e + 1, which each does only after it has
// finished reading epoch e.
//
// Every wait is bounded (kPeerWaitNs, 50 ms: a peer that is alive arrives
// within microseconds); on timeout the CTA records DEV_TIMEOUT_PEER in the
// device status word and returns, so a broken group fails fast.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "../../include/swq.h"
#include "allreduce.h"
#include "swq_device.cuh"

namespace swq {

namespace {

constexpr int AR_THREADS = 512;
constexpr uint64_t kPeerWaitNs = 50ull * 1000ull * 1000ull;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct ArArgs {
    float* data;          // in/out, this rank
    size_t n;             // elements
    int rank, world;
    size_t chunk;         // elements per CTA slice (multiple of 4)
    ArBuffer bufs[SWQ_AR_MAX_RANKS];  // every rank's buffer as mapped here
};

__global__ void __launch_bounds__(AR_THREADS) allreduce_kernel(const ArArgs a) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    const int b = blockIdx.x;
    const ArBuffer me = a.bufs[a.rank];
    if (threadIdx.x == 0) {
        s_epoch = ++me.epoch[b];
        s_ok = 1;
    }
    __syncthreads();
    const unsigned epoch = s_epoch;
    const size_t half = (epoch & 1u) ? me.half_elems : 0;
    const size_t lo = static_cast<size_t>(b) * a.chunk;
    const size_t hi = lo + a.chunk < a.n ? lo + a.chunk : a.n;
    const bool vec = (a.n % 4 == 0) && ((reinterpret_cast<uintptr_t>(a.data) & 15u) == 0);

    // 1. my slice into my buffer
    if (vec) {
        for (size_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * AR_THREADS)
            *reinterpret_cast<float4*>(me.data + half + i) = *reinterpret_cast<const float4*>(a.data + i);
    } else {
        for (size_t i = lo + threadIdx.x; i < hi; i += AR_THREADS) me.data[half + i] = a.data[i];
    }
    __syncthreads();
    // 2. publish
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(me.flag + b, epoch);
    }
    // 3. wait for every peer's slice b of this epoch
    if (threadIdx.x < a.world && threadIdx.x != a.rank) {
        const unsigned* f = a.bufs[threadIdx.x].flag + b;
        if (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
            const uint64_t t0 = globaltimer_ns();
            for (uint32_t i = 1;; ++i) {
                if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) break;
                if ((i & 63u) == 0 && globaltimer_ns() - t0 > kPeerWaitNs) {
                    atomicOr(&g_swq_dev_status, DEV_TIMEOUT_PEER);
                    s_ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;
    // 4. sum in rank order
    if (vec) {
        for (size_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * AR_THREADS) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < a.world; ++r) {
                const float4 v = __ldcv(reinterpret_cast<const float4*>(a.bufs[r].data + half + i));
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            *reinterpret_cast<float4*>(a.data + i) = acc;
        }
    } else {
        for (size_t i = lo + threadIdx.x; i < hi; i += AR_THREADS) {
            float acc = 0.f;
            for (int r = 0; r < a.world; ++r) acc += __ldcv(a.bufs[r].data + half + i);
            a.data[i] = acc;
        }
    }
}

}  // namespace

size_t allreduce_buffer_bytes(size_t max_elems) {
    return ar_header_bytes() + 2 * ((max_elems + 63) / 64 * 64) * sizeof(float);
}

size_t ar_header_bytes() { return 2 * SWQ_AR_MAX_CTAS * sizeof(unsigned); }

ArBuffer ar_view(void* base, size_t max_elems) {
    ArBuffer v;
    v.flag = static_cast<unsigned*>(base);
    v.epoch = v.flag + SWQ_AR_MAX_CTAS;
    v.data = reinterpret_cast<float*>(static_cast<uint8_t*>(base) + ar_header_bytes());
    v.half_elems = (max_elems + 63) / 64 * 64;
    return v;
}

cudaError_t allreduce_launch(const ArBuffer* bufs, int rank, int world, float* data, size_t n, int num_sms,
                             cudaStream_t s) {
    if (world < 1 || world > SWQ_AR_MAX_RANKS || rank < 0 || rank >= world) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    ArArgs a{};
    a.data = data;
    a.n = n;
    a.rank = rank;
    a.world = world;
    // about 2K elements per CTA, at most one CTA per SM (and per flag word)
    size_t ctas = (n + 2047) / 2048;
    const size_t cap = static_cast<size_t>(num_sms < SWQ_AR_MAX_CTAS ? num_sms : SWQ_AR_MAX_CTAS);
    if (ctas > cap) ctas = cap;
    if (ctas < 1) ctas = 1;
    a.chunk = ((n + ctas - 1) / ctas + 3) / 4 * 4;
    ctas = (n + a.chunk - 1) / a.chunk;
    for (int r = 0; r < world; ++r) a.bufs[r] = bufs[r];
    allreduce_kernel<<<static_cast<unsigned>(ctas), AR_THREADS, 0, s>>>(a);
    return cudaGetLastError();
}

SWQ_DEFINE_STATUS_FETCH(allreduce)

}  // namespace swq
