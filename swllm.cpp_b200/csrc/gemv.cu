// gemv.cu -- fused dequant + GEMV/small-M GEMM on GGUF blocks (sm_100a).
//
// Y[m][i] = sum_k X[m][k] * W[i][k] for m < M (M <= 8), i < N, W in GGUF
// blocks.  Replaces the per-format CPU routines cpu_matmul_transposed_*
// (src/tensor.h:570-1025) behind Compute::matmul_transposed_q
// (src/tensor.h:1212).
//
// Design (HBM-bound streaming):
//  * Persistent grid, CTA b owns a contiguous, balanced range of rows.
//  * Warp 8 is the producer: one lane streams row chunks of raw blocks into a
//    ring of shared-memory stages with cp.async.bulk (TMA bulk copies, no
//    multicast, L2 evict-first), completion on per-stage mbarriers.
//  * Warps 0-7 are consumers, one row per warp per stage.  A lane decodes one
//    "unit" (32 or 64 elements) from shared memory into packed small integers
//    and dots it with the activation row re-laid out as 16-bit fixed point
//    (per-32-element scale) with dp2a; per-part sums are scaled in fp32.
//  * The activation prep runs once per CTA (x -> shared memory) while the
//    first weight stages are already in flight.
//  * Programmatic dependent launch: weights (immutable inputs) are requested
//    before the previous kernel on the stream has finished; activations are
//    read only after griddepcontrol.wait.
//  * Every wait is bounded; on timeout the kernel records it in the device
//    status word, drains its own copies and returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <numeric>

#include "formats.cuh"
#include "gemv.h"
#include "swq_device.cuh"

namespace swq {

constexpr int kConsumerWarps = 8;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;

struct GemvParams {
    const uint8_t* W;
    const float* X;
    float* Y;
    int M, N, K;
    int nb;            // blocks per row
    int row_bytes;     // nb * BB
    int KC;            // blocks per chunk
    int nchunks;       // chunks per row
    int row_stride;    // bytes between rows inside a stage (16-aligned)
    int stage_bytes;   // kConsumerWarps * row_stride
    int stages;
    int bulk;          // 1: cp.async.bulk producer; 0: plain-load producer
    int refcpu;        // Q2_K reference-CPU activation order
    int early;         // weight prefetch before griddepcontrol.wait
    int x_vec;         // X is 16-byte aligned: float4 activation loads
    uint32_t off_xrec, off_xs, off_is, off_sx, off_h16, off_ring;  // smem offsets
};

// Layout helpers for the activation records.
template <int T>
struct XLayout {
    using F = Fmt<T>;
    static constexpr int C = F::UE / 8;  // 16-byte chunks per unit record
    static constexpr int L = 8 / C;      // records per 128-byte line
    __device__ static int rot(int u) { return (u / L) & (C - 1); }
};

template <int T, int MT>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvParams p) {
    using F = Fmt<T>;
    using XL = XLayout<T>;
    constexpr int UE = F::UE, PARTS = F::PARTS, UPB = F::UPB, QK = F::QK, BB = F::BB;
    constexpr int NW = UE / 4;  // q words per unit

    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + p.stages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + p.stages);
    uint8_t* xrec = smem + p.off_xrec;
    float* xs_arr = reinterpret_cast<float*>(smem + p.off_xs);
    int* is_arr = reinterpret_cast<int*>(smem + p.off_is);
    float* sx = reinterpret_cast<float*>(smem + p.off_sx);
    int* h16 = reinterpret_cast<int*>(smem + p.off_h16);
    uint8_t* ring = smem + p.off_ring;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = p.K / UE;  // units per row

    // Balanced contiguous row range of this CTA.
    const int G = gridDim.x, b = blockIdx.x;
    const int rlo = p.N / G, rex = p.N % G;
    const int r_begin = b * rlo + min(b, rex);
    const int r_end = r_begin + rlo + (b < rex ? 1 : 0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (!p.early) pdl_wait_primary();
        const uint64_t pol = l2_policy_evict_first();
        int it = 0;
        bool ok = true;
        for (int rg = r_begin; rg < r_end && ok; rg += kConsumerWarps) {
            const int rows = min(kConsumerWarps, r_end - rg);
            for (int ch = 0; ch < p.nchunks; ++ch, ++it) {
                const int s = it % p.stages;
                if (it >= p.stages) {
                    if (!mbar_wait_bounded(&empty[s], ((it / p.stages) - 1) & 1, DEV_TIMEOUT_EMPTY) ||
                        *abort_flag) {
                        ok = false;
                        *abort_flag = 1;
                        break;
                    }
                }
                const int kb0 = ch * p.KC;
                const int kc = min(p.KC, p.nb - kb0);
                const uint32_t bytes_row = static_cast<uint32_t>(kc * BB);
                uint8_t* dst = ring + static_cast<size_t>(s) * p.stage_bytes;
                const uint8_t* src = p.W + static_cast<size_t>(rg) * p.row_bytes +
                                     static_cast<size_t>(kb0) * BB;
                if (p.bulk) {
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&full[s], bytes_row * rows);
                        if (p.nchunks == 1) {
                            bulk_g2s(dst, src, bytes_row * rows, &full[s], pol);
                        } else {
                            for (int r = 0; r < rows; ++r)
                                bulk_g2s(dst + r * p.row_stride, src + static_cast<size_t>(r) * p.row_bytes,
                                         bytes_row, &full[s], pol);
                        }
                    }
                } else {
                    for (int r = 0; r < rows; ++r) {
                        const uint8_t* sr = src + static_cast<size_t>(r) * p.row_bytes;
                        uint8_t* dr = dst + r * p.row_stride;
                        for (uint32_t i = lane; i < bytes_row; i += 32) dr[i] = __ldg(sr + i);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[s]);
                }
            }
        }
        // Drain: make sure no bulk copy of this CTA is still writing shared memory.
        if (p.bulk && lane == 0) {
            const int issued = it;
            for (int s = 0; s < p.stages && s < issued; ++s) {
                const int last = issued - 1 - ((issued - 1 - s) % p.stages);  // last iteration on stage s
                mbar_wait_bounded(&full[s], (last / p.stages) & 1, DEV_TIMEOUT_DRAIN);
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    pdl_wait_primary();
    const int ctid = threadIdx.x;  // 0 .. 255
    constexpr int NCT = kConsumerWarps * 32;

    // Phase A: per 32-element block scale, 16-bit fixed point, per-16 sums;
    // scatter the fixed-point values into unit-order records.
    {
        const int k4 = p.K / 4;
        const int total = MT * k4;
        for (int f0 = 0; f0 < total; f0 += NCT) {
            const int f = f0 + ctid;  // total is a multiple of 8 (K % 32 == 0)
            const bool act = f < total;
            const int m = act ? f / k4 : 0;
            const int kk = act ? (f - m * k4) * 4 : 0;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (act && m < p.M) {
                const float* xp = p.X + static_cast<size_t>(m) * p.K + kk;
                if (p.x_vec) {
                    v = __ldg(reinterpret_cast<const float4*>(xp));
                } else {
                    v.x = __ldg(xp);
                    v.y = __ldg(xp + 1);
                    v.z = __ldg(xp + 2);
                    v.w = __ldg(xp + 3);
                }
            }
            float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
            a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
            a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
            a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
            const float inv = a > 0.f ? 32767.0f / a : 0.f;
            const float sc = a > 0.f ? a * (1.0f / 32767.0f) : 0.f;
            int xi[4];
            xi[0] = __float2int_rn(v.x * inv);
            xi[1] = __float2int_rn(v.y * inv);
            xi[2] = __float2int_rn(v.z * inv);
            xi[3] = __float2int_rn(v.w * inv);
#pragma unroll
            for (int i = 0; i < 4; ++i) xi[i] = max(-32767, min(32767, xi[i]));
            int s16 = xi[0] + xi[1] + xi[2] + xi[3];
            s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
            s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
            if (act) {
                if ((lane & 7) == 0) sx[m * (p.K / 32) + kk / 32] = sc;
                if ((lane & 3) == 0) h16[m * (p.K / 16) + kk / 16] = s16;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int k = kk + i;
                    const int kb = k / QK, kq = k % QK;
                    int cs[4], es[4];
                    const int nd = F::xdests(kq, p.refcpu != 0, cs, es);
                    for (int t = 0; t < nd; ++t) {
                        const int u = kb * UPB + cs[t];
                        const int e = es[t];
                        const int phys = ((e >> 3) + XL::rot(u)) & (XL::C - 1);
                        int16_t* rec = reinterpret_cast<int16_t*>(
                            xrec + (static_cast<size_t>(m) * units + u) * (2 * UE));
                        rec[phys * 8 + (e & 7)] = static_cast<int16_t>(xi[i]);
                    }
                }
            }
        }
    }
    named_bar_sync(1, NCT);
    // Phase B: per (m, unit, part) activation scale and integer sum.
    {
        const int total = MT * units * PARTS;
        for (int t = ctid; t < total; t += NCT) {
            const int m = t / (units * PARTS);
            const int r = t - m * units * PARTS;
            const int u = r / PARTS, part = r % PARTS;
            const int kb = u / UPB, c = u % UPB;
            const int xb = kb * (QK / 32) + F::part_xblock(c, part, p.refcpu != 0);
            const int hb = kb * (QK / 16) + F::part_half(c, part, p.refcpu != 0);
            int isum = h16[m * (p.K / 16) + hb];
            if (F::PE == 32) isum += h16[m * (p.K / 16) + hb + 1];
            xs_arr[t] = sx[m * (p.K / 32) + xb];
            is_arr[t] = isum;
        }
    }
    named_bar_sync(1, NCT);

    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.f;

    int it = 0;
    bool ok = true;
    for (int rg = r_begin; rg < r_end && ok; rg += kConsumerWarps) {
        const int rows = min(kConsumerWarps, r_end - rg);
        for (int ch = 0; ch < p.nchunks; ++ch, ++it) {
            const int s = it % p.stages;
            if (!mbar_wait_bounded(&full[s], (it / p.stages) & 1, DEV_TIMEOUT_FULL) || *abort_flag) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            if (warp < rows) {
                const int kb0 = ch * p.KC;
                const int kc = min(p.KC, p.nb - kb0);
                const uint8_t* rowp = ring + static_cast<size_t>(s) * p.stage_bytes + warp * p.row_stride;
                const int nu = kc * UPB;
                for (int uu = lane; uu < nu; uu += 32) {
                    const int kbl = uu / UPB, c = uu - kbl * UPB;
                    uint32_t q[NW];
                    float wd[PARTS], wm[PARTS];
                    F::decode(rowp + kbl * BB, c, q, wd, wm);
                    const int u = (kb0 + kbl) * UPB + c;
                    const int rot = XL::rot(u);
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const uint8_t* rec = xrec + (static_cast<size_t>(m) * units + u) * (2 * UE);
                        uint32_t P[UE / 2];
#pragma unroll
                        for (int j = 0; j < XL::C; ++j) {
                            const uint4 v = lds_u128(rec + 16 * ((j + rot) & (XL::C - 1)));
                            P[4 * j + 0] = v.x;
                            P[4 * j + 1] = v.y;
                            P[4 * j + 2] = v.z;
                            P[4 * j + 3] = v.w;
                        }
                        const int mi = (m * units + u) * PARTS;
                        float a = acc[m];
#pragma unroll
                        for (int pt = 0; pt < PARTS; ++pt) {
                            constexpr int WPP = NW / PARTS;  // q words per part
                            int S = 0;
#pragma unroll
                            for (int w = 0; w < WPP; ++w) {
                                const int wi = pt * WPP + w;
                                S = __dp2a_lo(static_cast<int>(P[2 * wi]), static_cast<int>(q[wi]), S);
                                S = __dp2a_hi(static_cast<int>(P[2 * wi + 1]), static_cast<int>(q[wi]), S);
                            }
                            const float xsv = xs_arr[mi + pt];
                            const int I = is_arr[mi + pt];
                            float t = wd[pt] * static_cast<float>(S - F::IOFF * I);
                            if (F::MIN) t = fmaf(-wm[pt], static_cast<float>(I), t);
                            a = fmaf(xsv, t, a);
                        }
                        acc[m] = a;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!ok) break;
        if (warp < rows) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                float v = acc[m];
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                v += __shfl_xor_sync(0xffffffffu, v, 8);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                if (lane == 0 && m < p.M) p.Y[static_cast<size_t>(m) * p.N + rg + warp] = v;
                acc[m] = 0.f;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

template <int T>
static size_t x_bytes(int MT, int K) {
    using F = Fmt<T>;
    const size_t units = K / F::UE;
    size_t b = 0;
    b += static_cast<size_t>(MT) * units * 2 * F::UE;          // records
    b += static_cast<size_t>(MT) * units * F::PARTS * 4 * 2;   // xs + isum
    b += static_cast<size_t>(MT) * (K / 32) * 4;               // sx
    b += static_cast<size_t>(MT) * (K / 16) * 4;               // h16
    return b;
}

static inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <int T, int MT>
static cudaError_t launch_t(const GemvLaunch& L, cudaStream_t stream) {
    using F = Fmt<T>;
    GemvParams p{};
    p.W = static_cast<const uint8_t*>(L.W);
    p.X = L.X;
    p.Y = L.Y;
    p.M = L.M;
    p.N = L.N;
    p.K = L.K;
    p.nb = L.K / F::QK;
    p.row_bytes = p.nb * F::BB;
    p.refcpu = L.refcpu;
    p.early = L.early;
    // every row start is then 16-byte aligned too (K % 32 == 0)
    p.x_vec = (reinterpret_cast<uintptr_t>(L.X) & 15u) == 0 ? 1 : 0;

    const bool base_al = (reinterpret_cast<uintptr_t>(L.W) & 15u) == 0;
    p.bulk = (base_al && (p.row_bytes % 16) == 0) ? 1 : 0;

    // Blocks per chunk: a multiple of the count that keeps chunk starts
    // 16-byte aligned, with stages near kStageTarget bytes.
    const int al_blocks = 16 / std::gcd(F::BB, 16);
    const int kStageTarget = 24 * 1024;
    int KC = kStageTarget / (kConsumerWarps * F::BB);
    KC = std::max(al_blocks, KC / al_blocks * al_blocks);
    if (KC >= p.nb) KC = p.nb;
    p.KC = KC;
    p.nchunks = (p.nb + KC - 1) / KC;
    p.row_stride = static_cast<int>(align_up(static_cast<uint32_t>(KC * F::BB), 16));
    p.stage_bytes = kConsumerWarps * p.row_stride;

    // Shared memory: barriers | x records | xs | isum | sx | h16 | ring.
    const int units = L.K / F::UE;
    uint32_t off = 0;
    off += 2 * 16 * 8 + 16;  // up to 16 stages x 2 barriers + abort flag
    off = align_up(off, 128);
    p.off_xrec = off;
    off += static_cast<uint32_t>(MT) * units * 2 * F::UE;
    p.off_xs = off;
    off += static_cast<uint32_t>(MT) * units * F::PARTS * 4;
    p.off_is = off;
    off += static_cast<uint32_t>(MT) * units * F::PARTS * 4;
    p.off_sx = off;
    off += static_cast<uint32_t>(MT) * (L.K / 32) * 4;
    p.off_h16 = off;
    off += static_cast<uint32_t>(MT) * (L.K / 16) * 4;
    off = align_up(off, 128);
    p.off_ring = off;

    const uint32_t smem_cap = static_cast<uint32_t>(L.smem_per_block_optin);
    const uint32_t sm_total = static_cast<uint32_t>(L.smem_per_sm);
    if (off + 2u * p.stage_bytes > smem_cap) return cudaErrorInvalidConfiguration;
    // Prefer two CTAs per SM with >= 3 stages, else one CTA with up to 8.
    int ctas_per_sm = 1;
    int stages = static_cast<int>((smem_cap - off) / p.stage_bytes);
    const uint32_t half = sm_total / 2 - 1024;  // per-CTA budget at 2 CTAs/SM
    if (half > off && static_cast<int>((half - off) / p.stage_bytes) >= 3) {
        ctas_per_sm = 2;
        stages = static_cast<int>((half - off) / p.stage_bytes);
    }
    stages = std::min(stages, 8);
    p.stages = stages;
    const uint32_t smem = off + static_cast<uint32_t>(stages) * p.stage_bytes;

    int grid = L.num_sms * ctas_per_sm;
    if (grid > L.N) grid = L.N;
    if (grid < 1) grid = 1;

    auto kern = gemv_kernel<T, MT>;
    // The attribute is per device: raise it once to the largest size seen.
    static thread_local int set_dev = -1;
    static thread_local uint32_t set_smem = 0;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev != set_dev || smem > set_smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_cap));
        if (e != cudaSuccess) return e;
        set_dev = dev;
        set_smem = smem_cap;
    }

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int T>
static cudaError_t launch_fmt(const GemvLaunch& L, cudaStream_t s) {
    if (L.M <= 1) return launch_t<T, 1>(L, s);
    if (L.M <= 2) return launch_t<T, 2>(L, s);
    if (L.M <= 4) return launch_t<T, 4>(L, s);
    return launch_t<T, 8>(L, s);
}

size_t gemv_smem_x_bytes(int type, int MT, int K) {
    switch (type) {
        case Q4_0: return x_bytes<Q4_0>(MT, K);
        case Q8_0: return x_bytes<Q8_0>(MT, K);
        case Q2_K: return x_bytes<Q2_K>(MT, K);
        case Q3_K: return x_bytes<Q3_K>(MT, K);
        case Q4_K: return x_bytes<Q4_K>(MT, K);
        case Q5_K: return x_bytes<Q5_K>(MT, K);
        case Q6_K: return x_bytes<Q6_K>(MT, K);
        default: return 0;
    }
}

cudaError_t gemv_launch(const GemvLaunch& L, cudaStream_t s) {
    switch (L.type) {
        case Q4_0: return launch_fmt<Q4_0>(L, s);
        case Q8_0: return launch_fmt<Q8_0>(L, s);
        case Q2_K: return launch_fmt<Q2_K>(L, s);
        case Q3_K: return launch_fmt<Q3_K>(L, s);
        case Q4_K: return launch_fmt<Q4_K>(L, s);
        case Q5_K: return launch_fmt<Q5_K>(L, s);
        case Q6_K: return launch_fmt<Q6_K>(L, s);
        default: return cudaErrorInvalidValue;
    }
}

SWQ_DEFINE_STATUS_FETCH(gemv)

}  // namespace swq
