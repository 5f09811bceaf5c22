// moe.cu -- mixture-of-experts routing, token sort, dispatch and combine on
// the device (sm_100a).
//
// The reference has no MoE forward (src/model.h:520-528 runs a dense FFN; the
// GGUF expert tensor names appear only at src/hf_loader.h:474-493), so these
// kernels implement the routing the MoE decoder shape calls for: an fp32
// router GEMV, the top-k logits per token, softmax over those k, a stable
// sort of the (token, slot) pairs by expert, and the weighted combine of the
// expert outputs.  Everything stays on the GPU: no count or offset goes back
// to the host, so a whole MoE layer can be captured in a CUDA graph.
//
// Expert parallelism (experts sharded over the GPUs of a group, one process
// per GPU) moves the routed rows over peer memory (CUDA IPC, NVLink /
// NVSwitch) instead of an NCCL all-to-all, whose split sizes would have to
// come back to the host first.  Per call, with epoch e counted on the device:
//   route    (1 CTA)  sort my pairs by global expert; store my per-expert
//                     counts into every rank's count matrix; publish e; wait
//                     (bounded) for every rank's counts; every rank then knows
//                     where each of its pairs lands in its expert's rows.
//   dispatch (G CTAs) copy each pair's token row straight into the receive
//                     buffer of the rank that owns its expert (peer stores),
//                     with a (source, slot) tag; publish e per CTA; CTA b
//                     waits for CTA b of every source.
//   [the caller's grouped expert GEMMs on the received rows]
//   return   (G CTAs) copy each expert output row back into its source's
//                     return buffer; publish e per CTA.
//   reduce   (G CTAs) wait for every CTA of every rank's return; then
//                     y[t] = sum_j w[t,j] * out[t,j].
// A rank writes into a peer's buffers for epoch e + 1 only after its own
// reduce of epoch e has seen every peer's returned rows, which each peer
// sends only after it has finished reading its receive buffer of epoch e: one
// copy of each buffer suffices.  Every wait gives up after kPeerWaitNs (1 s)
// and records DEV_TIMEOUT_PEER.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/swq.h"
#include "moe.h"
#include "swq_device.cuh"

namespace swq {

namespace {

// A peer rank may reach a call later than this one by its host-side launch
// work (including the first, lazily loaded launch of a kernel), so the bound
// is a second rather than the all-reduce's 50 ms.
constexpr uint64_t kPeerWaitNs = 1000ull * 1000ull * 1000ull;
constexpr int ROUTE_WARPS = 8;
constexpr int ROUTE_EPC = 16;       // experts per CTA of the router GEMV
constexpr int SORT_THREADS = 1024;  // the sort runs in one CTA, 32 warps
constexpr int SORT_WARPS = SORT_THREADS / 32;
constexpr int EP_THREADS = 512;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Wait until *f (written by another GPU) reaches `epoch`; false on timeout.
__device__ bool wait_epoch(const unsigned* f, unsigned epoch) {
    if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (static_cast<int>(ld_acquire_sys(f) - epoch) >= 0) return true;
        if ((i & 63u) == 0 && globaltimer_ns() - t0 > kPeerWaitNs) {
            atomicOr(&g_swq_dev_status, DEV_TIMEOUT_PEER);
            return false;
        }
    }
}

// ---------------------------------------------------------------- router
// logits[t][e] = sum_h Wr[e][h] * X[t][h] (fp32).  CTA (tile of TT tokens,
// ROUTE_EPC experts); the tokens' rows are staged in shared memory and each
// warp reduces its experts' dot products across lanes in a fixed order.
template <int TT, bool VEC>
__global__ void __launch_bounds__(ROUTE_WARPS * 32)
    router_logits_kernel(const float* __restrict__ Wr, const float* __restrict__ X, float* __restrict__ logits,
                         int T, int E, int H) {
    extern __shared__ __align__(16) float xs[];  // [TT][H]
    const int t0 = blockIdx.x * TT;
    const int nt = min(TT, T - t0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < TT * H; i += blockDim.x) {
        const int t = i / H;
        xs[i] = t < nt ? X[static_cast<size_t>(t0 + t) * H + (i - t * H)] : 0.f;
    }
    __syncthreads();
    const int e_end = min(E, (blockIdx.y + 1) * ROUTE_EPC);
    for (int e = blockIdx.y * ROUTE_EPC + warp; e < e_end; e += ROUTE_WARPS) {
        const float* w = Wr + static_cast<size_t>(e) * H;
        float acc[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = 0.f;
        if (VEC) {
            for (int h = 4 * lane; h < H; h += 128) {
                const float4 wv = __ldg(reinterpret_cast<const float4*>(w + h));
#pragma unroll
                for (int t = 0; t < TT; ++t) {
                    const float4 xv = *reinterpret_cast<const float4*>(xs + t * H + h);
                    acc[t] = fmaf(wv.x, xv.x, acc[t]);
                    acc[t] = fmaf(wv.y, xv.y, acc[t]);
                    acc[t] = fmaf(wv.z, xv.z, acc[t]);
                    acc[t] = fmaf(wv.w, xv.w, acc[t]);
                }
            }
        } else {
            for (int h = lane; h < H; h += 32) {
                const float wv = __ldg(w + h);
#pragma unroll
                for (int t = 0; t < TT; ++t) acc[t] = fmaf(wv, xs[t * H + h], acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
        }
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < TT; ++t)
                if (t < nt) logits[static_cast<size_t>(t0 + t) * E + e] = acc[t];
        }
    }
}

// One warp per token: the k largest logits (ties: the lower expert id first;
// NaN ranks as -inf), in descending order, and softmax over them:
// w_j = exp(l_j - l_0) / sum_i exp(l_i - l_0), the sum taken left to right.
__global__ void __launch_bounds__(256) topk_softmax_kernel(const float* __restrict__ logits, int T, int E, int k,
                                                           int* __restrict__ ids, float* __restrict__ wts) {
    constexpr int PER = SWQ_MOE_MAX_EXPERTS / 32;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    const float* l = logits + static_cast<size_t>(t) * E;
    float v[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        float x = e < E ? l[e] : -INFINITY;
        v[i] = (x != x) ? -INFINITY : x;
    }
    unsigned taken = 0;
    float sv = 0.f;
    int si = 0;
    for (int j = 0; j < k; ++j) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((taken >> i) & 1u) && (v[i] > bv || (v[i] == bv && e < bi))) {
                bv = v[i];
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        if (lane == j) {
            sv = bv;
            si = bi;
        }
    }
    const float vmax = __shfl_sync(0xffffffffu, sv, 0);
    const float ex = lane < k ? expf(sv - vmax) : 0.f;
    float sum = 0.f;
    for (int j = 0; j < k; ++j) sum += __shfl_sync(0xffffffffu, ex, j);
    if (lane < k) {
        ids[static_cast<size_t>(t) * k + lane] = si;
        wts[static_cast<size_t>(t) * k + lane] = ex / sum;
    }
}

// ---------------------------------------------------------------- sort
// Stable counting sort of P pairs by expert id, in one CTA of 1024 threads.
// Warp w owns the pairs [w*seg, (w+1)*seg); cnt[w][e] counts its pairs of
// expert e, then becomes the first output row of those pairs.  Rows are
// expert-major, and within an expert in pair order.  A pair whose id is not
// in [0, E) gets row -1 and is left out (DEV_BAD_ID).
//   cnt    shared, SORT_WARPS * E ints;  wsum shared, 32 ints
//   start  E + 1 ints (any memory): expert e's first row; start[E] = rows
//   sorted rows ints: the pair of each row;  prow P ints: the row of each pair
__device__ void sort_pairs(const int* __restrict__ ids, int P, int E, int* cnt, int* wsum, int* start,
                           int* __restrict__ sorted, int* __restrict__ prow) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < SORT_WARPS * E; i += blockDim.x) cnt[i] = 0;
    __syncthreads();
    const int seg = (P + SORT_WARPS - 1) / SORT_WARPS;
    const int p0 = min(P, warp * seg), p1 = min(P, p0 + seg);
    int* my = cnt + warp * E;
    bool bad = false;
    for (int base = p0; base < p1; base += 32) {
        const int p = base + lane;
        int e = p < p1 ? ids[p] : -1;
        const bool ok = p < p1 && e >= 0 && e < E;
        bad |= (p < p1) && !ok;
        e = ok ? e : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        if (ok && lane == 31 - __clz(peers)) my[e] += __popc(peers);
        __syncwarp();
    }
    if (bad) atomicOr(&g_swq_dev_status, DEV_BAD_ID);
    __syncthreads();
    // expert totals, exclusive scan over experts (thread e), then per-warp bases
    const int e = threadIdx.x;
    int tot = 0;
    if (e < E)
        for (int w = 0; w < SORT_WARPS; ++w) tot += cnt[w * E + e];
    int incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int v = wsum[lane];
        int s = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        wsum[lane] = s - v;
    }
    __syncthreads();
    if (e < E) {
        int run = incl - tot + wsum[warp];
        start[e] = run;
        for (int w = 0; w < SORT_WARPS; ++w) {
            const int c = cnt[w * E + e];
            cnt[w * E + e] = run;
            run += c;
        }
        if (e == E - 1) start[E] = run;
    }
    __syncthreads();
    for (int base = p0; base < p1; base += 32) {
        const int p = base + lane;
        int e2 = p < p1 ? ids[p] : -1;
        const bool ok = p < p1 && e2 >= 0 && e2 < E;
        e2 = ok ? e2 : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e2);
        const int r = ok ? my[e2] + __popc(peers & lanemask_lt()) : -1;
        __syncwarp();
        if (ok && lane == 31 - __clz(peers)) my[e2] += __popc(peers);
        __syncwarp();
        if (p < p1) {
            prow[p] = r;
            if (ok) sorted[r] = p;
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(SORT_THREADS) sort_kernel(const int* ids, int P, int E, int* offsets, int* sorted,
                                                            int* prow) {
    extern __shared__ int cnt[];
    __shared__ int wsum[32];
    sort_pairs(ids, P, E, cnt, wsum, offsets, sorted, prow);
}

// X_sorted[r] = X[sorted[r] / k] for the rows r < offsets[E].
template <bool VEC>
__global__ void __launch_bounds__(256) gather_kernel(const float* __restrict__ X, const int* __restrict__ sorted,
                                                     const int* __restrict__ offsets, int E, int P, int k, int H,
                                                     float* __restrict__ Xs) {
    const int rows = min(P, offsets[E]);
    const int warps = gridDim.x * 8;
    for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += warps) {
        const float* src = X + static_cast<size_t>(sorted[r] / k) * H;
        float* dst = Xs + static_cast<size_t>(r) * H;
        if (VEC) {
            for (int h = 4 * (threadIdx.x & 31); h < H; h += 128)
                *reinterpret_cast<float4*>(dst + h) = __ldg(reinterpret_cast<const float4*>(src + h));
        } else {
            for (int h = threadIdx.x & 31; h < H; h += 32) dst[h] = __ldg(src + h);
        }
    }
}

// Y[t][h] = (accumulate ? Y[t][h] : 0) + sum_j w[t,j] * Ys[prow[t*k+j]][h],
// one fused multiply-add per slot, j = 0 .. k-1; slots with row -1 add nothing.
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ Ys, const int* __restrict__ prow,
                                                      const float* __restrict__ w, int T, int k, int H,
                                                      float* __restrict__ Y, int accumulate) {
    const int64_t n = static_cast<int64_t>(T) * H;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i / H);
        const int h = static_cast<int>(i - static_cast<int64_t>(t) * H);
        float acc = accumulate ? Y[i] : 0.f;
        for (int j = 0; j < k; ++j) {
            const int r = prow[t * k + j];
            if (r >= 0) acc = fmaf(w[t * k + j], Ys[static_cast<size_t>(r) * H + h], acc);
        }
        Y[i] = acc;
    }
}

// ---------------------------------------------------------------- expert parallel
struct EpArgs {
    EpView bufs[SWQ_EP_MAX_RANKS];  // every rank's buffer as mapped here
    EpView me;
    int rank, world, E, el, k, H, cap;
};

// Sorts this rank's pairs, exchanges the per-expert counts and computes every
// pair's destination row.  One CTA of SORT_THREADS.
__global__ void __launch_bounds__(SORT_THREADS) ep_route_kernel(const EpArgs a, const int* __restrict__ ids, int T) {
    extern __shared__ int sm[];
    int* cnt = sm;                                 // [SORT_WARPS][E]
    int* start = cnt + SORT_WARPS * a.E;           // [E + 1] my sorted rows per expert
    int* dest = start + a.E + 1;                   // [E] first destination row of my pairs of e
    __shared__ int wsum[32];
    __shared__ int obase[SWQ_EP_MAX_RANKS];
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    const EpView me = a.me;
    const int P = T * a.k;
    if (threadIdx.x == 0) {
        s_epoch = ++me.epoch[0];
        s_ok = 1;
        me.meta[EP_META_P] = P;
        me.meta[EP_META_T] = T;
    }
    sort_pairs(ids, P, a.E, cnt, wsum, start, me.spair, me.prow);  // ends with __syncthreads
    const unsigned epoch = s_epoch;
    // my per-expert counts into row `rank` of every rank's count matrix
    for (int i = threadIdx.x; i < a.world * a.E; i += blockDim.x) {
        const int d = i / a.E, e = i - d * a.E;
        a.bufs[d].cm[a.rank * a.E + e] = start[e + 1] - start[e];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int d = 0; d < a.world; ++d) st_release_sys(a.bufs[d].cflag + a.rank, epoch);
    }
    if (threadIdx.x < a.world && !wait_epoch(me.cflag + threadIdx.x, epoch)) s_ok = 0;
    __syncthreads();
    if (!s_ok) {
        if (threadIdx.x == 0) me.meta[EP_META_OK] = 0;
        return;
    }
    // totals per expert over the sources, exclusive scan within each owner
    const int e = threadIdx.x;
    int tot = 0, before = 0;
    if (e < a.E) {
        for (int s = 0; s < a.world; ++s) {
            const int c = __ldcv(me.cm + s * a.E + e);
            if (s < a.rank) before += c;
            tot += c;
        }
    }
    // inclusive scan of tot over all experts (E <= 1024 threads)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int v = wsum[lane];
        int s = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += u;
        }
        wsum[lane] = s - v;
    }
    __syncthreads();
    const int excl = incl - tot + wsum[warp];  // rows of experts 0 .. e-1, all owners
    // each owner's rows start at 0: subtract the rows of the owners before it
    if (e < a.E && e % a.el == 0) obase[e / a.el] = excl;
    __syncthreads();
    if (e < a.E) {
        const int base = excl - obase[e / a.el];  // expert e's first row on its owner
        dest[e] = base + before;                  // ... and the first one of my pairs
        if (e / a.el == a.rank) {
            me.loff[e - a.rank * a.el] = base;
            if (e == (a.rank + 1) * a.el - 1) me.loff[a.el] = base + tot;
        }
    }
    __syncthreads();
    // destination row of each of my sorted rows
    const int rows = start[a.E];
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {
        const int p = me.spair[i];
        const int ex = ids[p];
        me.drow[i] = dest[ex] + (i - start[ex]);
    }
    if (threadIdx.x == 0) {
        me.meta[EP_META_ROWS] = rows;
        me.meta[EP_META_OK] = 1;
    }
}

template <bool VEC>
__device__ __forceinline__ void copy_row(float* dst, const float* src, int H, int lane) {
    if (VEC) {
        for (int h = 4 * lane; h < H; h += 128)
            *reinterpret_cast<float4*>(dst + h) = __ldcv(reinterpret_cast<const float4*>(src + h));
    } else {
        for (int h = lane; h < H; h += 32) dst[h] = __ldcv(src + h);
    }
}

// Copies my sorted rows into their owners' receive buffers; CTA b copies the
// b-th slice, one warp per row, then publishes and waits for CTA b of every
// rank.  Launched with exactly EP_CTAS CTAs.
template <bool VEC>
__global__ void __launch_bounds__(EP_THREADS) ep_dispatch_kernel(const EpArgs a, const int* __restrict__ ids,
                                                                 const float* __restrict__ X) {
    __shared__ int s_ok;
    const EpView me = a.me;
    const unsigned epoch = me.epoch[0];
    const bool ok = me.meta[EP_META_OK] != 0;
    if (threadIdx.x == 0) s_ok = ok ? 1 : 0;
    const int rows = ok ? me.meta[EP_META_ROWS] : 0;
    const int per = (rows + EP_CTAS - 1) / EP_CTAS;
    const int r0 = min(rows, static_cast<int>(blockIdx.x) * per), r1 = min(rows, r0 + per);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = r0 + warp; i < r1; i += EP_THREADS / 32) {
        const int p = me.spair[i];
        const int d = ids[p] / a.el;
        const int row = me.drow[i];
        copy_row<VEC>(a.bufs[d].rbuf + static_cast<size_t>(row) * a.H, X + static_cast<size_t>(p / a.k) * a.H, a.H,
                      lane);
        if (lane == 0) a.bufs[d].rtag[row] = make_int2(a.rank, i);
    }
    __syncthreads();
    if (!ok) return;
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int d = 0; d < a.world; ++d) st_release_sys(a.bufs[d].dflag + a.rank * EP_CTAS + blockIdx.x, epoch);
    }
    if (threadIdx.x < a.world && !wait_epoch(me.dflag + threadIdx.x * EP_CTAS + blockIdx.x, epoch)) s_ok = 0;
    __syncthreads();
    if (!s_ok && threadIdx.x == 0) me.meta[EP_META_OK] = 0;
}

// Returns the expert outputs Yr (rows as received) to their sources and
// publishes each CTA's part.  Exactly EP_CTAS CTAs.  No wait here: a CTA that
// waited for the other CTAs of its own grid could wait for CTAs that are not
// resident yet.
template <bool VEC>
__global__ void __launch_bounds__(EP_THREADS) ep_return_kernel(const EpArgs a, const float* __restrict__ Yr) {
    const EpView me = a.me;
    const unsigned epoch = me.epoch[0];
    const bool ok = me.meta[EP_META_OK] != 0;
    const int R = ok ? min(max(me.loff[a.el], 0), a.cap) : 0;
    const int per = (R + EP_CTAS - 1) / EP_CTAS;
    const int r0 = min(R, static_cast<int>(blockIdx.x) * per), r1 = min(R, r0 + per);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = r0 + warp; r < r1; r += EP_THREADS / 32) {
        const int2 tag = __ldcv(me.rtag + r);
        copy_row<VEC>(a.bufs[tag.x].ret + static_cast<size_t>(tag.y) * a.H, Yr + static_cast<size_t>(r) * a.H, a.H,
                      lane);
    }
    __syncthreads();
    if (!ok) return;
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int d = 0; d < a.world; ++d) st_release_sys(a.bufs[d].rflag + a.rank * EP_CTAS + blockIdx.x, epoch);
    }
}

// Waits for every CTA of every rank's return, then y[t] = (accumulate ? y[t] :
// 0) + sum_j w[t,j] * out[t,j] with one fused multiply-add per slot, j = 0 ..
// k-1 (slots of bad ids add nothing).
__global__ void __launch_bounds__(EP_THREADS) ep_reduce_kernel(const EpArgs a, const float* __restrict__ w,
                                                               float* __restrict__ Y, int accumulate) {
    __shared__ int s_ok;
    const EpView me = a.me;
    const unsigned epoch = me.epoch[0];
    const bool ok = me.meta[EP_META_OK] != 0;
    if (threadIdx.x == 0) s_ok = ok ? 1 : 0;
    __syncthreads();
    if (!ok) return;
    for (int j = threadIdx.x; j < a.world * EP_CTAS; j += blockDim.x) {
        if (!*reinterpret_cast<volatile int*>(&s_ok)) break;
        if (!wait_epoch(me.rflag + j, epoch)) s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) {
        if (threadIdx.x == 0) me.meta[EP_META_OK] = 0;
        return;
    }
    const int T = me.meta[EP_META_T];
    const int64_t n = static_cast<int64_t>(T) * a.H;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i / a.H);
        const int h = static_cast<int>(i - static_cast<int64_t>(t) * a.H);
        float acc = accumulate ? Y[i] : 0.f;
        for (int j = 0; j < a.k; ++j) {
            const int slot = me.prow[t * a.k + j];
            if (slot >= 0) acc = fmaf(w[t * a.k + j], __ldcv(me.ret + static_cast<size_t>(slot) * a.H + h), acc);
        }
        Y[i] = acc;
    }
}

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

template <typename K>
cudaError_t smem_optin(K kern, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

int gather_grid(int64_t rows, int num_sms) {
    const int64_t g = (rows + 7) / 8;
    return static_cast<int>(g < 1 ? 1 : (g > 8 * num_sms ? 8 * num_sms : g));
}

}  // namespace

// ---------------------------------------------------------------- host side

cudaError_t moe_router_launch(const float* Wr, const float* X, float* logits, int T, int E, int H, int k, int* ids,
                              float* w, int smem_max, cudaStream_t s) {
    const bool vec = H % 4 == 0 && (reinterpret_cast<uintptr_t>(Wr) & 15u) == 0;
    // tokens per CTA: 8 while their rows fit the shared memory
    int tt = 8;
    while (tt > 1 && static_cast<size_t>(tt) * H * sizeof(float) > static_cast<size_t>(smem_max)) tt >>= 1;
    const size_t smem = static_cast<size_t>(tt) * H * sizeof(float);
    if (smem > static_cast<size_t>(smem_max)) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>((T + tt - 1) / tt), static_cast<unsigned>((E + ROUTE_EPC - 1) / ROUTE_EPC));
    cudaError_t e = cudaSuccess;
#define SWQ_ROUTE_CASE(TT)                                                                     \
    case TT:                                                                                   \
        if (vec) {                                                                             \
            if ((e = smem_optin(router_logits_kernel<TT, true>, smem)) != cudaSuccess) return e; \
            router_logits_kernel<TT, true><<<grid, ROUTE_WARPS * 32, smem, s>>>(Wr, X, logits, T, E, H); \
        } else {                                                                               \
            if ((e = smem_optin(router_logits_kernel<TT, false>, smem)) != cudaSuccess) return e; \
            router_logits_kernel<TT, false><<<grid, ROUTE_WARPS * 32, smem, s>>>(Wr, X, logits, T, E, H); \
        }                                                                                      \
        break;
    switch (tt) {
        SWQ_ROUTE_CASE(8)
        SWQ_ROUTE_CASE(4)
        SWQ_ROUTE_CASE(2)
        SWQ_ROUTE_CASE(1)
        default: return cudaErrorInvalidValue;
    }
#undef SWQ_ROUTE_CASE
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    topk_softmax_kernel<<<(T + 7) / 8, 256, 0, s>>>(logits, T, E, k, ids, w);
    return cudaGetLastError();
}

cudaError_t moe_sort_launch(const int* ids, int P, int E, int* offsets, int* sorted, int* prow, cudaStream_t s) {
    const size_t smem = static_cast<size_t>(SORT_WARPS) * E * sizeof(int);
    cudaError_t e = smem_optin(sort_kernel, smem);
    if (e != cudaSuccess) return e;
    sort_kernel<<<1, SORT_THREADS, smem, s>>>(ids, P, E, offsets, sorted, prow);
    return cudaGetLastError();
}

cudaError_t moe_gather_launch(const float* X, const int* sorted, const int* offsets, int E, int P, int k, int H,
                              float* Xs, int num_sms, cudaStream_t s) {
    const bool vec = H % 4 == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(Xs) & 15u) == 0;
    const int grid = gather_grid(P, num_sms);
    if (vec) gather_kernel<true><<<grid, 256, 0, s>>>(X, sorted, offsets, E, P, k, H, Xs);
    else gather_kernel<false><<<grid, 256, 0, s>>>(X, sorted, offsets, E, P, k, H, Xs);
    return cudaGetLastError();
}

cudaError_t moe_combine_launch(const float* Ys, const int* prow, const float* w, int T, int k, int H, float* Y,
                               int accumulate, int num_sms, cudaStream_t s) {
    const int64_t n = static_cast<int64_t>(T) * H;
    int64_t g = (n + 255) / 256;
    if (g > 8 * num_sms) g = 8 * num_sms;
    if (g < 1) g = 1;
    combine_kernel<<<static_cast<int>(g), 256, 0, s>>>(Ys, prow, w, T, k, H, Y, accumulate);
    return cudaGetLastError();
}

size_t ep_header_bytes() {
    return align256((SWQ_EP_MAX_RANKS + 2 * SWQ_EP_MAX_RANKS * EP_CTAS + 1 + EP_META_WORDS) * sizeof(unsigned));
}

EpView ep_view(void* base, const EpShape& sh) {
    EpView v{};
    uint8_t* b = static_cast<uint8_t*>(base);
    v.cflag = reinterpret_cast<unsigned*>(b);
    v.dflag = v.cflag + SWQ_EP_MAX_RANKS;
    v.rflag = v.dflag + SWQ_EP_MAX_RANKS * EP_CTAS;
    v.epoch = v.rflag + SWQ_EP_MAX_RANKS * EP_CTAS;
    v.meta = reinterpret_cast<int*>(v.epoch + 1);
    size_t off = ep_header_bytes();
    const size_t pt = static_cast<size_t>(sh.max_tokens) * sh.k;
    const size_t cap = pt * sh.world;
    const int el = sh.E / sh.world;
    v.cm = reinterpret_cast<int*>(b + off);
    off += align256(sizeof(int) * SWQ_EP_MAX_RANKS * sh.E);
    v.loff = reinterpret_cast<int*>(b + off);
    off += align256(sizeof(int) * (el + 1));
    v.spair = reinterpret_cast<int*>(b + off);
    off += align256(sizeof(int) * pt);
    v.prow = reinterpret_cast<int*>(b + off);
    off += align256(sizeof(int) * pt);
    v.drow = reinterpret_cast<int*>(b + off);
    off += align256(sizeof(int) * pt);
    v.rtag = reinterpret_cast<int2*>(b + off);
    off += align256(sizeof(int2) * cap);
    v.rbuf = reinterpret_cast<float*>(b + off);
    off += align256(sizeof(float) * cap * sh.H);
    v.ret = reinterpret_cast<float*>(b + off);
    return v;
}

size_t ep_buffer_bytes(const EpShape& sh) {
    const EpView v = ep_view(nullptr, sh);
    const size_t pt = static_cast<size_t>(sh.max_tokens) * sh.k;
    return reinterpret_cast<size_t>(v.ret) + align256(sizeof(float) * pt * sh.H);
}

static EpArgs ep_args(const EpView* bufs, int rank, const EpShape& sh) {
    EpArgs a{};
    for (int r = 0; r < sh.world; ++r) a.bufs[r] = bufs[r];
    a.me = bufs[rank];
    a.rank = rank;
    a.world = sh.world;
    a.E = sh.E;
    a.el = sh.E / sh.world;
    a.k = sh.k;
    a.H = sh.H;
    a.cap = sh.max_tokens * sh.k * sh.world;
    return a;
}

cudaError_t ep_dispatch_launch(const EpView* bufs, int rank, const EpShape& sh, const int* ids, const float* X, int T,
                               cudaStream_t s) {
    const EpArgs a = ep_args(bufs, rank, sh);
    const size_t smem = sizeof(int) * (static_cast<size_t>(SORT_WARPS) * sh.E + 2 * sh.E + 1);
    cudaError_t e = smem_optin(ep_route_kernel, smem);
    if (e != cudaSuccess) return e;
    ep_route_kernel<<<1, SORT_THREADS, smem, s>>>(a, ids, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const bool vec = sh.H % 4 == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0;
    if (vec) ep_dispatch_kernel<true><<<EP_CTAS, EP_THREADS, 0, s>>>(a, ids, X);
    else ep_dispatch_kernel<false><<<EP_CTAS, EP_THREADS, 0, s>>>(a, ids, X);
    return cudaGetLastError();
}

cudaError_t ep_combine_launch(const EpView* bufs, int rank, const EpShape& sh, const float* Yr, const float* w,
                              float* Y, int accumulate, cudaStream_t s) {
    const EpArgs a = ep_args(bufs, rank, sh);
    const bool vec = sh.H % 4 == 0 && (reinterpret_cast<uintptr_t>(Yr) & 15u) == 0;
    if (vec) ep_return_kernel<true><<<EP_CTAS, EP_THREADS, 0, s>>>(a, Yr);
    else ep_return_kernel<false><<<EP_CTAS, EP_THREADS, 0, s>>>(a, Yr);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    ep_reduce_kernel<<<EP_CTAS, EP_THREADS, 0, s>>>(a, w, Y, accumulate);
    return cudaGetLastError();
}

SWQ_DEFINE_STATUS_FETCH(moe)

}  // namespace swq
