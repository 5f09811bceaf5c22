// api.cu -- the extern "C" boundary of libswq (declared in include/swq.h).
//
// Argument checks, per-device properties, options, status words and the
// host-buffer context.  All compute is in the kernels (gemv.cu, dequant.cu,
// gemm_tc.cu); nothing here computes on the CPU.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/swq.h"
#include "allreduce.h"
#include "moe.h"
#include "decode.h"
#include "prefill.h"
#include "qkv_extras.h"
#include "gemm_tc.h"
#include "gdn.h"
#include "gemv.h"
#include "gemv_kqm.h"

namespace {

thread_local std::string g_last_error;

std::atomic<int> g_opt_q2k_refcpu{1};
std::atomic<int> g_opt_early_prefetch{1};
std::atomic<int> g_opt_gemv_max_m{8};
std::atomic<int> g_opt_gemm_tc{1};
std::atomic<int> g_opt_tc_min_m{5};
std::atomic<int> g_opt_gemv_smem_kb{0};
std::atomic<int> g_opt_gemv_stage_kb{0};
std::atomic<int> g_opt_gemv_ctas{0};
std::atomic<int> g_opt_gemv_fp32{1};
std::atomic<int> g_opt_gemv_imma{2};
std::atomic<int> g_opt_kqm_max_m{16};
std::atomic<int> g_opt_kqm_table_kb{0};
std::atomic<int> g_opt_kqm_group{0};
std::atomic<int> g_opt_attn_form{3};

swq_status fail(swq_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

swq_status cuda_fail(cudaError_t e, const char* where) {
    g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return SWQ_ERR_CUDA;
}

struct TypeInfo {
    int qk, bb;
};

bool type_info(int t, TypeInfo* ti) {
    switch (t) {
        case SWQ_TYPE_Q4_0: *ti = {32, 18}; return true;
        case SWQ_TYPE_Q8_0: *ti = {32, 34}; return true;
        case SWQ_TYPE_Q2_K: *ti = {256, 84}; return true;
        case SWQ_TYPE_Q3_K: *ti = {256, 110}; return true;
        case SWQ_TYPE_Q4_K: *ti = {256, 144}; return true;
        case SWQ_TYPE_Q5_K: *ti = {256, 176}; return true;
        case SWQ_TYPE_Q6_K: *ti = {256, 210}; return true;
        default: return false;
    }
}

std::mutex g_dev_mu;
std::map<int, swq::DeviceInfo> g_dev;

swq_status current_device(swq::DeviceInfo* out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_dev_mu);
    auto it = g_dev.find(dev);
    if (it == g_dev.end()) {
        swq::DeviceInfo d;
        d.device = dev;
        if ((e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.smem_per_block_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) !=
                cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) !=
                cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        it = g_dev.emplace(dev, d).first;
    }
    *out = it->second;
    if (out->cc_major != 10)
        return fail(SWQ_ERR_UNSUPPORTED, "libswq is built for sm_100a (B200); device " + std::to_string(dev) +
                                             " is sm_" + std::to_string(out->cc_major) +
                                             std::to_string(out->cc_minor));
    return SWQ_OK;
}

// Largest activation-row group the GEMV kernel takes for this K: the per-CTA
// activation copy must leave room for at least three weight stages.
int gemv_group_rows(int type, int K, int max_m) {
    const size_t budget = 120 * 1024;
    for (int g : {8, 4, 2, 1}) {
        if (g > max_m && g != 1) continue;
        if (swq::gemv_smem_x_bytes(type, g, K, g_opt_gemv_fp32 != 0) <= budget) return g;
    }
    return 0;
}

swq_status check_gemm_args(int type, const void* W, const float* X, const float* Y, int M, int N, int K,
                           TypeInfo* ti) {
    if (!type_info(type, ti)) return fail(SWQ_ERR_BAD_TYPE, "type " + std::to_string(type) + " is not on this path");
    if (M < 0 || N < 0 || K < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (K % ti->qk != 0)
        return fail(SWQ_ERR_BAD_SHAPE, "K=" + std::to_string(K) + " is not a multiple of " + std::to_string(ti->qk));
    if (M == 0 || N == 0 || K == 0) return SWQ_OK;
    if (!W || !X || !Y) return fail(SWQ_ERR_NULL_PTR, "null W, X or Y");
    return SWQ_OK;
}

// The batched K-quant GEMV (2 <= M <= SWQ_OPT_GEMV_BATCH_MAX_M rows of Q4_K or
// Q6_K) takes this call.
bool kqm_takes(int type, const void* W, int M, int N, int K, const swq::DeviceInfo& dev) {
    return g_opt_kqm_max_m >= 2 &&
           swq::gemv_kqm_supported(type, W, M, N, K, g_opt_kqm_max_m, dev.num_sms, dev.smem_per_block_optin);
}

// Batched K-quant GEMV with its scratch from the caller (ws) or, when ws is
// null, from libswq's stream-ordered pool.
swq_status kqm_run(int type, const void* W, const float* X, float* Y, int M, int N, int K, const swq::ActArgs& act,
                   const swq::DeviceInfo& dev, cudaStream_t s, void* ws = nullptr, size_t ws_bytes = 0) {
    const size_t need = swq::gemv_kqm_workspace_bytes(type, M, N, K, dev.num_sms, dev.smem_per_block_optin);
    if (ws != nullptr) {
        if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
            return fail(SWQ_ERR_BAD_ARG, "workspace not 256-byte aligned");
        if (ws_bytes < need)
            return fail(SWQ_ERR_BAD_ARG, "workspace of " + std::to_string(ws_bytes) + " bytes, this call needs " +
                                             std::to_string(need));
        cudaError_t e = swq::gemv_kqm_launch(type, W, X, Y, M, N, K, act, g_opt_early_prefetch, dev.num_sms,
                                             dev.smem_per_block_optin, ws, ws_bytes, s);
        return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "batched K-quant GEMV launch (caller workspace)");
    }
    void* buf = nullptr;
    cudaError_t e = swq::scratch_alloc(&buf, need, s);
    if (e != cudaSuccess) return cuda_fail(e, "batched K-quant GEMV scratch");
    e = swq::gemv_kqm_launch(type, W, X, Y, M, N, K, act, g_opt_early_prefetch, dev.num_sms, dev.smem_per_block_optin,
                             buf, need, s);
    cudaError_t e2 = swq::scratch_free(buf, s);
    if (e != cudaSuccess) return cuda_fail(e, "batched K-quant GEMV launch");
    return e2 == cudaSuccess ? SWQ_OK : cuda_fail(e2, "batched K-quant GEMV scratch free");
}

// Y = X . W^T through the GEMV kernel, groups of up to max_m rows of X.
swq_status gemm_gemv_groups(int type, const void* W, const float* X, float* Y, int M, int N, int K, int max_m,
                            const swq::DeviceInfo& dev, cudaStream_t s, const swq::ActArgs& act = swq::ActArgs{}) {
    const int g = gemv_group_rows(type, K, std::max(1, max_m));
    if (g == 0) return fail(SWQ_ERR_BAD_SHAPE, "K=" + std::to_string(K) + " exceeds the GEMV activation buffer");
    const int ld = act.ld > 0 ? act.ld : K;
    for (int m0 = 0; m0 < M; m0 += g) {
        swq::GemvLaunch L{};
        L.type = type;
        L.W = W;
        L.X = X + static_cast<size_t>(m0) * ld;
        L.Y = Y + static_cast<size_t>(m0) * N;
        L.act = act.kind;
        L.R = act.R ? act.R + static_cast<size_t>(m0) * K : nullptr;
        L.normw = act.normw;
        L.eps = act.eps;
        L.sum_out = act.sum_out ? act.sum_out + static_cast<size_t>(m0) * K : nullptr;
        L.ld = ld;
        L.M = std::min(g, M - m0);
        L.N = N;
        L.K = K;
        L.refcpu = g_opt_q2k_refcpu;
        L.early = g_opt_early_prefetch;
        L.num_sms = dev.num_sms;
        L.smem_per_block_optin = dev.smem_per_block_optin;
        L.smem_per_sm = dev.smem_per_sm;
        L.smem_kb = g_opt_gemv_smem_kb;
        L.stage_kb = g_opt_gemv_stage_kb;
        L.ctas_per_sm = g_opt_gemv_ctas;
        L.xf = g_opt_gemv_fp32;
        L.imma = g_opt_gemv_imma;
        cudaError_t e = swq::gemv_launch(L, s);
        if (e != cudaSuccess) return cuda_fail(e, "GEMV launch");
    }
    return SWQ_OK;
}

}  // namespace

extern "C" {

const char* swq_status_string(swq_status s) {
    switch (s) {
        case SWQ_OK: return "ok";
        case SWQ_ERR_BAD_TYPE: return "bad type";
        case SWQ_ERR_BAD_SHAPE: return "bad shape";
        case SWQ_ERR_NULL_PTR: return "null pointer";
        case SWQ_ERR_CUDA: return "cuda error";
        case SWQ_ERR_TIMEOUT: return "device wait timed out";
        case SWQ_ERR_UNSUPPORTED: return "unsupported";
        case SWQ_ERR_BAD_ARG: return "bad argument";
    }
    return "unknown status";
}

const char* swq_last_error(void) { return g_last_error.c_str(); }

size_t swq_type_size(int t) {
    TypeInfo ti;
    return type_info(t, &ti) ? static_cast<size_t>(ti.bb) : 0;
}

size_t swq_block_size(int t) {
    TypeInfo ti;
    return type_info(t, &ti) ? static_cast<size_t>(ti.qk) : 0;
}

swq_status swq_set_option(int option, int value) {
    switch (option) {
        case SWQ_OPT_Q2K_REFERENCE_CPU_ORDER:
            if (value != 0 && value != 1) return fail(SWQ_ERR_BAD_ARG, "option value must be 0 or 1");
            g_opt_q2k_refcpu = value;
            return SWQ_OK;
        case SWQ_OPT_EARLY_WEIGHT_PREFETCH:
            if (value != 0 && value != 1) return fail(SWQ_ERR_BAD_ARG, "option value must be 0 or 1");
            g_opt_early_prefetch = value;
            swq::gemm_tc_set_early_prefetch(value);
            return SWQ_OK;
        case SWQ_OPT_GEMV_MAX_M:
            if (value < 0 || value > 8) return fail(SWQ_ERR_BAD_ARG, "GEMV max M must be in 0..8");
            g_opt_gemv_max_m = value;
            return SWQ_OK;
        case SWQ_OPT_TENSOR_CORE_GEMM:
            if (value != 0 && value != 1) return fail(SWQ_ERR_BAD_ARG, "option value must be 0 or 1");
            g_opt_gemm_tc = value;
            return SWQ_OK;
        case SWQ_OPT_TENSOR_CORE_MIN_M:
            if (value < 2) return fail(SWQ_ERR_BAD_ARG, "tensor-core minimum M must be >= 2");
            g_opt_tc_min_m = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_SMEM_KB:
            if (value < 0 || value > 1024) return fail(SWQ_ERR_BAD_ARG, "GEMV shared memory must be 0..1024 KB");
            g_opt_gemv_smem_kb = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_STAGE_KB:
            if (value < 0 || value > 1024) return fail(SWQ_ERR_BAD_ARG, "GEMV stage size must be 0..1024 KB");
            g_opt_gemv_stage_kb = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_CTAS_PER_SM:
            if (value < 0 || value > 4) return fail(SWQ_ERR_BAD_ARG, "GEMV CTAs per SM must be 0..4");
            g_opt_gemv_ctas = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_FP32_ACT:
            if (value != 0 && value != 1) return fail(SWQ_ERR_BAD_ARG, "option value must be 0 or 1");
            g_opt_gemv_fp32 = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_INT_MMA:
            if (value < 0 || value > 2) return fail(SWQ_ERR_BAD_ARG, "option value must be 0, 1 or 2");
            g_opt_gemv_imma = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_BATCH_MAX_M:
            if (value < 0) return fail(SWQ_ERR_BAD_ARG, "option value must be >= 0");
            g_opt_kqm_max_m = value;
            return SWQ_OK;
        case SWQ_OPT_GEMV_BATCH_TABLE_KB:
            if (value != 0 && (value < 8 || value > 160))
                return fail(SWQ_ERR_BAD_ARG, "option value must be 0 or 8..160");
            g_opt_kqm_table_kb = value;
            swq::gemv_kqm_tune(g_opt_kqm_table_kb, g_opt_kqm_group);
            return SWQ_OK;
        case SWQ_OPT_GEMV_BATCH_GROUP:
            if (value != 0 && value != 1 && value != 2 && value != 4 && value != 8 && value != 16)
                return fail(SWQ_ERR_BAD_ARG, "option value must be 0, 1, 2, 4, 8 or 16");
            g_opt_kqm_group = value;
            swq::gemv_kqm_tune(g_opt_kqm_table_kb, g_opt_kqm_group);
            return SWQ_OK;
        case SWQ_OPT_PREFILL_ATTENTION:
            if (value < 0 || value > 3) return fail(SWQ_ERR_BAD_ARG, "option value must be 0, 1, 2 or 3");
            g_opt_attn_form = value;
            return SWQ_OK;
        default:
            return fail(SWQ_ERR_BAD_ARG, "unknown option " + std::to_string(option));
    }
}

int swq_get_option(int option) {
    switch (option) {
        case SWQ_OPT_Q2K_REFERENCE_CPU_ORDER: return g_opt_q2k_refcpu;
        case SWQ_OPT_EARLY_WEIGHT_PREFETCH: return g_opt_early_prefetch;
        case SWQ_OPT_GEMV_MAX_M: return g_opt_gemv_max_m;
        case SWQ_OPT_TENSOR_CORE_GEMM: return g_opt_gemm_tc;
        case SWQ_OPT_TENSOR_CORE_MIN_M: return g_opt_tc_min_m;
        case SWQ_OPT_GEMV_SMEM_KB: return g_opt_gemv_smem_kb;
        case SWQ_OPT_GEMV_STAGE_KB: return g_opt_gemv_stage_kb;
        case SWQ_OPT_GEMV_CTAS_PER_SM: return g_opt_gemv_ctas;
        case SWQ_OPT_GEMV_FP32_ACT: return g_opt_gemv_fp32;
        case SWQ_OPT_GEMV_INT_MMA: return g_opt_gemv_imma;
        case SWQ_OPT_GEMV_BATCH_MAX_M: return g_opt_kqm_max_m;
        case SWQ_OPT_GEMV_BATCH_TABLE_KB: return g_opt_kqm_table_kb;
        case SWQ_OPT_GEMV_BATCH_GROUP: return g_opt_kqm_group;
        case SWQ_OPT_PREFILL_ATTENTION: return g_opt_attn_form;
        default: return -1;
    }
}

swq_status swq_dequant(int type, const void* blocks, float* out, int64_t n, swq_stream_t stream) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return fail(SWQ_ERR_BAD_TYPE, "type " + std::to_string(type) + " is not on this path");
    if (n < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative n");
    const int64_t nblocks = n / ti.qk;
    if (nblocks == 0) return SWQ_OK;
    if (!blocks || !out) return fail(SWQ_ERR_NULL_PTR, "null blocks or out");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    cudaError_t e = swq::dequant_launch(type, blocks, out, nblocks, dev.num_sms,
                                        reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
    return SWQ_OK;
}

swq_status swq_gemm(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                    swq_stream_t stream) {
    TypeInfo ti;
    swq_status st = check_gemm_args(type, W, X, Y, M, N, K, &ti);
    if (st != SWQ_OK || M == 0 || N == 0) return st;
    swq::DeviceInfo dev;
    if ((st = current_device(&dev)) != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(Y, 0, sizeof(float) * static_cast<size_t>(M) * N, s);
        return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    const int max_m = g_opt_gemv_max_m;
    if (kqm_takes(type, W, M, N, K, dev)) return kqm_run(type, W, X, Y, M, N, K, swq::ActArgs{}, dev, s);
    if (M >= g_opt_tc_min_m && g_opt_gemm_tc &&
        swq::gemm_tc_supported(type, W, M, N, K, g_opt_q2k_refcpu)) {
        cudaError_t e = swq::gemm_tc_launch(type, W, X, Y, M, N, K, g_opt_q2k_refcpu, dev.num_sms, s);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM launch");
        return SWQ_OK;
    }
    return gemm_gemv_groups(type, W, X, Y, M, N, K, max_m, dev, s);
}

// swq_act -> kernel arguments, with the checks every act-taking entry makes.
static swq_status parse_act(const swq_act* act, int K, swq::ActArgs* a) {
    if (!act) return SWQ_OK;
    if (act->kind != SWQ_ACT_NONE && act->kind != SWQ_ACT_RMSNORM && act->kind != SWQ_ACT_SWIGLU)
        return fail(SWQ_ERR_BAD_ARG, "unknown activation prologue " + std::to_string(act->kind));
    a->kind = act->kind;
    if (a->kind == SWQ_ACT_RMSNORM) {
        if (!act->norm_w) return fail(SWQ_ERR_NULL_PTR, "RMSNORM needs norm_w");
        if (!(act->eps >= 0.f)) return fail(SWQ_ERR_BAD_ARG, "eps must be >= 0");
        a->R = act->residual;
        a->normw = act->norm_w;
        a->eps = act->eps;
        a->sum_out = act->sum_out;
    } else if (a->kind == SWQ_ACT_SWIGLU) {
        a->ld = act->ld > 0 ? act->ld : 2 * K;
        if (a->ld < 2 * K) return fail(SWQ_ERR_BAD_SHAPE, "SWIGLU row stride below 2K");
    }
    return SWQ_OK;
}

swq_status swq_gemm_act(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                        const swq_act* act, int flags, swq_stream_t stream) {
    TypeInfo ti;
    swq_status st = check_gemm_args(type, W, X, Y, M, N, K, &ti);
    if (st != SWQ_OK || M == 0 || N == 0) return st;
    if (flags & ~SWQ_GEMM_NOALLOC) return fail(SWQ_ERR_BAD_ARG, "unknown flags");
    swq::ActArgs a;
    if ((st = parse_act(act, K, &a)) != SWQ_OK) return st;
    const bool noalloc = (flags & SWQ_GEMM_NOALLOC) != 0;
    if (noalloc && static_cast<int64_t>(M) * K > SWQ_GEMM_NOALLOC_MAX_X_ELEMS)
        return fail(SWQ_ERR_BAD_SHAPE, "swq_gemm_act: M*K exceeds the fixed scratch");
    swq::DeviceInfo dev;
    if ((st = current_device(&dev)) != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) return fail(SWQ_ERR_BAD_SHAPE, "swq_gemm_act needs K > 0");
    if (!noalloc && kqm_takes(type, W, M, N, K, dev)) return kqm_run(type, W, X, Y, M, N, K, a, dev, s);
    if (M >= g_opt_tc_min_m && g_opt_gemm_tc && swq::gemm_tc_supported(type, W, M, N, K, g_opt_q2k_refcpu)) {
        cudaError_t e = noalloc ? swq::gemm_tc_launch_noalloc(type, W, X, Y, M, N, K, g_opt_q2k_refcpu, dev.num_sms,
                                                              s, a)
                                : swq::gemm_tc_launch(type, W, X, Y, M, N, K, g_opt_q2k_refcpu, dev.num_sms, s, a);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM launch");
        return SWQ_OK;
    }
    return gemm_gemv_groups(type, W, X, Y, M, N, K, g_opt_gemv_max_m, dev, s, a);
}

size_t swq_gemm_workspace_bytes(int type, int M, int N, int K) {
    TypeInfo ti;
    if (!type_info(type, &ti) || M <= 0 || N <= 0 || K <= 0 || K % ti.qk != 0) return 0;
    swq::DeviceInfo dev;
    if (current_device(&dev) != SWQ_OK) return 0;
    // the batched K-quant GEMV (W's alignment is checked again at the call)
    if (kqm_takes(type, reinterpret_cast<const void*>(256), M, N, K, dev))
        return swq::gemv_kqm_workspace_bytes(type, M, N, K, dev.num_sms, dev.smem_per_block_optin);
    if (M < g_opt_tc_min_m || !g_opt_gemm_tc) return 0;  // the GEMV kernel needs no scratch
    return swq::gemm_tc_workspace_bytes(M, N, K, dev.num_sms);
}

swq_status swq_gemm_act_ws(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                           const swq_act* act, void* workspace, size_t workspace_bytes, swq_stream_t stream) {
    TypeInfo ti;
    swq_status st = check_gemm_args(type, W, X, Y, M, N, K, &ti);
    if (st != SWQ_OK || M == 0 || N == 0) return st;
    swq::ActArgs a;
    if ((st = parse_act(act, K, &a)) != SWQ_OK) return st;
    if (K == 0) return fail(SWQ_ERR_BAD_SHAPE, "swq_gemm_act_ws needs K > 0");
    swq::DeviceInfo dev;
    if ((st = current_device(&dev)) != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (kqm_takes(type, W, M, N, K, dev)) {
        if (!workspace) return fail(SWQ_ERR_NULL_PTR, "swq_gemm_act_ws: this call needs a workspace");
        return kqm_run(type, W, X, Y, M, N, K, a, dev, s, workspace, workspace_bytes);
    }
    if (M >= g_opt_tc_min_m && g_opt_gemm_tc && swq::gemm_tc_supported(type, W, M, N, K, g_opt_q2k_refcpu)) {
        const size_t need = swq::gemm_tc_workspace_bytes(M, N, K, dev.num_sms);
        if (!workspace) return fail(SWQ_ERR_NULL_PTR, "swq_gemm_act_ws: this call needs a workspace");
        if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
            return fail(SWQ_ERR_BAD_ARG, "swq_gemm_act_ws: workspace not 256-byte aligned");
        if (workspace_bytes < need)
            return fail(SWQ_ERR_BAD_ARG, "swq_gemm_act_ws: workspace of " + std::to_string(workspace_bytes) +
                                             " bytes, this call needs " + std::to_string(need));
        cudaError_t e = swq::gemm_tc_launch_ws(type, W, X, Y, M, N, K, g_opt_q2k_refcpu, dev.num_sms, s, a,
                                               workspace, workspace_bytes);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM launch (caller workspace)");
        return SWQ_OK;
    }
    return gemm_gemv_groups(type, W, X, Y, M, N, K, g_opt_gemv_max_m, dev, s, a);
}

swq_status swq_gemm_noalloc(int type, const void* W, const float* X, float* Y, int M, int N, int K,
                            swq_stream_t stream) {
    TypeInfo ti;
    swq_status st = check_gemm_args(type, W, X, Y, M, N, K, &ti);
    if (st != SWQ_OK || M == 0 || N == 0) return st;
    if (static_cast<int64_t>(M) * K > SWQ_GEMM_NOALLOC_MAX_X_ELEMS)
        return fail(SWQ_ERR_BAD_SHAPE, "swq_gemm_noalloc: M*K = " + std::to_string(static_cast<int64_t>(M) * K) +
                                           " exceeds its fixed scratch of " +
                                           std::to_string(SWQ_GEMM_NOALLOC_MAX_X_ELEMS) + " elements");
    swq::DeviceInfo dev;
    if ((st = current_device(&dev)) != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(Y, 0, sizeof(float) * static_cast<size_t>(M) * N, s);
        return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    const int max_m = g_opt_gemv_max_m;
    if (M >= g_opt_tc_min_m && g_opt_gemm_tc &&
        swq::gemm_tc_supported(type, W, M, N, K, g_opt_q2k_refcpu)) {
        cudaError_t e = swq::gemm_tc_launch_noalloc(type, W, X, Y, M, N, K, g_opt_q2k_refcpu, dev.num_sms, s);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core GEMM launch (fixed scratch)");
        return SWQ_OK;
    }
    return gemm_gemv_groups(type, W, X, Y, M, N, K, max_m, dev, s);
}

swq_status swq_grouped_gemm(int type, const void* const* W_experts, const int* expert_offsets, const float* X_sorted,
                            float* Y, int n_experts, int total_rows, int N, int K, swq_stream_t stream) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return fail(SWQ_ERR_BAD_TYPE, "type " + std::to_string(type) + " is not on this path");
    if (n_experts < 0 || total_rows < 0 || N < 0 || K < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (K % ti.qk != 0)
        return fail(SWQ_ERR_BAD_SHAPE, "K=" + std::to_string(K) + " is not a multiple of " + std::to_string(ti.qk));
    if (n_experts > 4095) return fail(SWQ_ERR_BAD_SHAPE, "n_experts above 4095");
    if (n_experts == 0 || total_rows == 0 || N == 0) return SWQ_OK;
    if (!W_experts || !expert_offsets || !X_sorted || !Y) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(Y, 0, sizeof(float) * static_cast<size_t>(total_rows) * N, s);
        return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    cudaError_t e = swq::gemm_tc_grouped_launch(type, W_experts, expert_offsets, X_sorted, Y, n_experts, total_rows,
                                                N, K, g_opt_q2k_refcpu, dev.num_sms, s);
    if (e != cudaSuccess) return cuda_fail(e, "grouped GEMM launch");
    return SWQ_OK;
}

swq_status swq_grouped_gemv(int type, const void* const* W_experts, const int* expert_offsets, const float* X_sorted,
                            float* Y, int n_experts, int total_rows, int N, int K, swq_stream_t stream) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return fail(SWQ_ERR_BAD_TYPE, "type " + std::to_string(type) + " is not on this path");
    if (n_experts < 0 || total_rows < 0 || N < 0 || K < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (K % ti.qk != 0)
        return fail(SWQ_ERR_BAD_SHAPE, "K=" + std::to_string(K) + " is not a multiple of " + std::to_string(ti.qk));
    if (n_experts > 65535) return fail(SWQ_ERR_BAD_SHAPE, "n_experts above 65535");
    if (n_experts == 0 || total_rows == 0 || N == 0) return SWQ_OK;
    if (!W_experts || !expert_offsets || !X_sorted || !Y) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(Y, 0, sizeof(float) * static_cast<size_t>(total_rows) * N, s);
        return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    cudaError_t e = swq::grouped_gemv_launch(type, W_experts, expert_offsets, X_sorted, Y, n_experts, total_rows, N,
                                             K, g_opt_q2k_refcpu, dev.smem_per_block_optin, s);
    if (e != cudaSuccess) return cuda_fail(e, "grouped GEMV launch");
    return SWQ_OK;
}

static swq_status grouped_matmul_impl(int type, const void* const* W_experts, const void* W_all,
                                      const int* expert_offsets, const float* X_sorted, float* Y, int n_experts,
                                      int total_rows, int N, int K, int mean_rows, swq_stream_t stream) {
    TypeInfo ti;
    if (!type_info(type, &ti)) return fail(SWQ_ERR_BAD_TYPE, "type " + std::to_string(type) + " is not on this path");
    if (n_experts < 0 || total_rows < 0 || N < 0 || K < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (K % ti.qk != 0)
        return fail(SWQ_ERR_BAD_SHAPE, "K=" + std::to_string(K) + " is not a multiple of " + std::to_string(ti.qk));
    if (n_experts > 4095) return fail(SWQ_ERR_BAD_SHAPE, "n_experts above 4095");
    if (n_experts == 0 || total_rows == 0 || N == 0) return SWQ_OK;
    if ((!W_experts && !W_all) || !expert_offsets || !X_sorted || !Y)
        return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(Y, 0, sizeof(float) * static_cast<size_t>(total_rows) * N, s);
        return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "cudaMemsetAsync");
    }
    cudaError_t e;
    if (mean_rows <= 4)
        e = swq::grouped_gemv_launch(type, W_experts, expert_offsets, X_sorted, Y, n_experts, total_rows, N, K,
                                     g_opt_q2k_refcpu, dev.smem_per_block_optin, s, true, W_all);
    else
        e = swq::gemm_tc_grouped_launch(type, W_experts, expert_offsets, X_sorted, Y, n_experts, total_rows, N, K,
                                        g_opt_q2k_refcpu, dev.num_sms, s, mean_rows, expert_offsets + n_experts,
                                        W_all);
    if (e != cudaSuccess) return cuda_fail(e, "grouped matmul launch");
    return SWQ_OK;
}

swq_status swq_grouped_matmul(int type, const void* const* W_experts, const int* expert_offsets, const float* X_sorted,
                              float* Y, int n_experts, int total_rows, int N, int K, int mean_rows,
                              swq_stream_t stream) {
    if (!W_experts) return fail(SWQ_ERR_NULL_PTR, "null expert table");
    return grouped_matmul_impl(type, W_experts, nullptr, expert_offsets, X_sorted, Y, n_experts, total_rows, N, K,
                               mean_rows, stream);
}

swq_status swq_grouped_matmul_stacked(int type, const void* W_all, const int* expert_offsets, const float* X_sorted,
                                      float* Y, int n_experts, int total_rows, int N, int K, int mean_rows,
                                      swq_stream_t stream) {
    if (!W_all) return fail(SWQ_ERR_NULL_PTR, "null expert tensor");
    return grouped_matmul_impl(type, nullptr, W_all, expert_offsets, X_sorted, Y, n_experts, total_rows, N, K,
                               mean_rows, stream);
}

// ---- decode step -------------------------------------------------------------

static swq_status launch_status(cudaError_t e, const char* what) {
    return e == cudaSuccess ? SWQ_OK : cuda_fail(e, what);
}

swq_status swq_rmsnorm(float* out, const float* x, const float* w, int n, float eps, int rows, swq_stream_t stream) {
    if (n < 0 || rows < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (n == 0 || rows == 0) return SWQ_OK;
    if (!out || !x || !w) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::rmsnorm_launch(out, const_cast<float*>(x), nullptr, w, n, eps, rows,
                                             reinterpret_cast<cudaStream_t>(stream)),
                         "rmsnorm launch");
}

swq_status swq_add_rmsnorm(float* out, float* x, const float* y, const float* w, int n, float eps, int rows,
                           swq_stream_t stream) {
    if (n < 0 || rows < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (n == 0 || rows == 0) return SWQ_OK;
    if (!out || !x || !y || !w) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::rmsnorm_launch(out, x, y, w, n, eps, rows, reinterpret_cast<cudaStream_t>(stream)),
                         "add_rmsnorm launch");
}

swq_status swq_rope_kv(float* q, const float* k, const float* v, float* k_cache, float* v_cache, const int* pos,
                       const float* freqs, int q_dim, int kv_dim, int head_dim, int rope_dim, int neox, int rows,
                       int max_seq, int ldq, int ldk, int ldv, swq_stream_t stream) {
    ldq = ldq ? ldq : q_dim;
    ldk = ldk ? ldk : kv_dim;
    ldv = ldv ? ldv : kv_dim;
    if (ldq < q_dim || ldk < kv_dim || ldv < kv_dim) return fail(SWQ_ERR_BAD_SHAPE, "row stride below row size");
    if (head_dim <= 0 || rope_dim <= 0 || rope_dim > head_dim || rope_dim % 2 || q_dim % head_dim ||
        kv_dim % head_dim || rows < 0 || max_seq <= 0)
        return fail(SWQ_ERR_BAD_SHAPE, "inconsistent RoPE dimensions");
    if (rows == 0) return SWQ_OK;
    if (!q || !k || !v || !k_cache || !v_cache || !pos || !freqs) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::rope_kv_launch(q, k, v, k_cache, v_cache, pos, freqs, q_dim, kv_dim, head_dim, rope_dim,
                                             neox, rows, max_seq, ldq, ldk, ldv, dev.num_sms,
                                             reinterpret_cast<cudaStream_t>(stream)),
                         "rope launch");
}

swq_status swq_qkv_bias_norm(float* q, float* k, float* v, const float* bq, const float* bk, const float* bv,
                              const float* q_norm, const float* k_norm, int q_dim, int kv_dim, int head_dim,
                              float eps, int rows, int ldq, int ldk, int ldv, swq_stream_t stream) {
    ldq = ldq ? ldq : q_dim;
    ldk = ldk ? ldk : kv_dim;
    ldv = ldv ? ldv : kv_dim;
    if (head_dim <= 0 || q_dim <= 0 || kv_dim <= 0 || q_dim % head_dim || kv_dim % head_dim || rows < 0)
        return fail(SWQ_ERR_BAD_SHAPE, "q/k/v extras: inconsistent head dimensions");
    if (ldq < q_dim || ldk < kv_dim || ldv < kv_dim) return fail(SWQ_ERR_BAD_SHAPE, "row stride below row size");
    if (rows == 0 || !(bq || bk || bv || q_norm || k_norm)) return SWQ_OK;  // nothing to do
    if (((bq || q_norm) && !q) || ((bk || k_norm) && !k) || (bv && !v))
        return fail(SWQ_ERR_NULL_PTR, "null q / k / v with a bias or norm for it");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::qkv_extras_launch(q, k, v, bq, bk, bv, q_norm, k_norm, q_dim, kv_dim, head_dim, eps,
                                                rows, ldq, ldk, ldv, reinterpret_cast<cudaStream_t>(stream)),
                         "q/k/v extras launch");
}

swq_status swq_gdn_step(const float* qkv, int ld_qkv, const float* z, const float* beta, const float* alpha,
                        const float* dt, const float* ssm_a, const float* conv_w, const float* norm_w, float* state,
                        float* conv_state, float* y, int rows, int n_k_heads, int n_v_heads, int key_head_dim,
                        int value_head_dim, int conv_width, swq_stream_t stream) {
    if (rows < 0 || n_k_heads <= 0 || n_v_heads <= 0 || key_head_dim <= 0 || value_head_dim <= 0 ||
        conv_width < 0)
        return fail(SWQ_ERR_BAD_SHAPE, "gdn step: non-positive head count or size");
    if (value_head_dim > swq::gdn_max_head_dim() || key_head_dim > 16384)
        return fail(SWQ_ERR_BAD_SHAPE, "gdn step: head dimension above the kernel's limit (value 1024, key 16384)");
    const long long qkv_dim = 2LL * n_k_heads * key_head_dim + 1LL * n_v_heads * value_head_dim;
    if (ld_qkv == 0) ld_qkv = static_cast<int>(qkv_dim);
    if (ld_qkv < qkv_dim) return fail(SWQ_ERR_BAD_SHAPE, "gdn step: q/k/v row stride below its size");
    if (rows == 0) return SWQ_OK;
    if (!qkv || !state || !y || (conv_w && conv_width > 0 && !conv_state))
        return fail(SWQ_ERR_NULL_PTR, "gdn step: null q/k/v, state, output or conv history");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::gdn_step_launch(qkv, ld_qkv, z, beta, alpha, dt, ssm_a, conv_w, norm_w, state,
                                              conv_state, y, rows, n_k_heads, n_v_heads, key_head_dim,
                                              value_head_dim, conv_width, reinterpret_cast<cudaStream_t>(stream)),
                         "gdn step launch");
}

// ---- prefill (rows m = s * seq_len + p: token p of sequence s at pos0 + p) ----

static swq_status prefill_rows(int num_seqs, int seq_len, int pos0, int max_seq, int* rows) {
    if (num_seqs < 0 || seq_len < 0 || pos0 < 0 || max_seq <= 0)
        return fail(SWQ_ERR_BAD_SHAPE, "prefill: negative size or empty cache");
    if (static_cast<long long>(pos0) + seq_len > max_seq)
        return fail(SWQ_ERR_BAD_SHAPE, "prefill: pos0 + seq_len exceeds the cache (max_seq)");
    const long long m = static_cast<long long>(num_seqs) * seq_len;
    if (m > 0x7fffffffLL) return fail(SWQ_ERR_BAD_SHAPE, "prefill: too many rows");
    *rows = static_cast<int>(m);
    return SWQ_OK;
}

swq_status swq_rope_kv_prefill(float* q, const float* k, const float* v, float* k_cache, float* v_cache, int pos0,
                               int seq_len, const float* freqs, int q_dim, int kv_dim, int head_dim, int rope_dim,
                               int neox, int num_seqs, int max_seq, int ldq, int ldk, int ldv, swq_stream_t stream) {
    ldq = ldq ? ldq : q_dim;
    ldk = ldk ? ldk : kv_dim;
    ldv = ldv ? ldv : kv_dim;
    if (ldq < q_dim || ldk < kv_dim || ldv < kv_dim) return fail(SWQ_ERR_BAD_SHAPE, "row stride below row size");
    if (head_dim <= 0 || rope_dim <= 0 || rope_dim > head_dim || rope_dim % 2 || q_dim <= 0 || kv_dim <= 0 ||
        q_dim % head_dim || kv_dim % head_dim)
        return fail(SWQ_ERR_BAD_SHAPE, "inconsistent RoPE dimensions");
    int rows = 0;
    swq_status st = prefill_rows(num_seqs, seq_len, pos0, max_seq, &rows);
    if (st != SWQ_OK || rows == 0) return st;
    if (!q || !k || !v || !k_cache || !v_cache || !freqs) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::rope_kv_prefill_launch(q, k, v, k_cache, v_cache, pos0, seq_len, freqs, q_dim, kv_dim,
                                                     head_dim, rope_dim, neox, rows, max_seq, ldq, ldk, ldv,
                                                     reinterpret_cast<cudaStream_t>(stream)),
                         "prefill rope launch");
}

swq_status swq_attention_prefill(float* out, const float* q, const float* k_cache, const float* v_cache, int pos0,
                                 int seq_len, int num_heads, int num_kv_heads, int head_dim, int num_seqs,
                                 int max_seq, int ldq, int ldo, swq_stream_t stream) {
    if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads ||
        (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256))
        return fail(SWQ_ERR_BAD_SHAPE, "prefill attention: head_dim 32/64/128/256, kv heads dividing query heads");
    const int row = num_heads * head_dim;
    ldq = ldq ? ldq : row;
    ldo = ldo ? ldo : row;
    if (ldq < row || ldo < row) return fail(SWQ_ERR_BAD_SHAPE, "row stride below row size");
    int rows = 0;
    swq_status st = prefill_rows(num_seqs, seq_len, pos0, max_seq, &rows);
    if (st != SWQ_OK || rows == 0) return st;
    if (!out || !q || !k_cache || !v_cache) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::attention_prefill_launch(out, q, k_cache, v_cache, pos0, seq_len, rows, num_heads,
                                                       num_kv_heads, head_dim, max_seq, ldq, ldo,
                                                       reinterpret_cast<cudaStream_t>(stream), g_opt_attn_form),
                         "prefill attention launch");
}

static int attention_splits_for(int rows, int num_kv_heads, int max_seq) {
    swq::DeviceInfo dev;
    if (current_device(&dev) != SWQ_OK) return 1;
    return swq::attention_splits(rows, num_kv_heads, max_seq, dev.num_sms);
}

size_t swq_attention_workspace_bytes(int num_heads, int num_kv_heads, int head_dim, int rows, int max_seq) {
    if (num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || rows <= 0 || max_seq <= 0) return 0;
    return swq::attention_workspace(num_heads, num_kv_heads, head_dim, rows,
                                    attention_splits_for(rows, num_kv_heads, max_seq));
}

swq_status swq_attention_decode(float* out, const float* q, const float* k_cache, const float* v_cache, const int* pos,
                                void* workspace, size_t workspace_bytes, int num_heads, int num_kv_heads, int head_dim,
                                int rows, int max_seq, int ldq, swq_stream_t stream) {
    if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || head_dim % 32 || head_dim > 256 ||
        rows < 0 || max_seq <= 0 || (num_heads / num_kv_heads) > 8 || ((num_heads / num_kv_heads) & (num_heads / num_kv_heads - 1)))
        return fail(SWQ_ERR_BAD_SHAPE, "attention: head_dim 64/128/256, 1/2/4/8 query heads per kv head");
    if (rows == 0) return SWQ_OK;
    if (!out || !q || !k_cache || !v_cache || !pos || !workspace) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    const size_t need = swq_attention_workspace_bytes(num_heads, num_kv_heads, head_dim, rows, max_seq);
    if (workspace_bytes < need) return fail(SWQ_ERR_BAD_ARG, "attention workspace too small");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    ldq = ldq ? ldq : num_heads * head_dim;
    if (ldq < num_heads * head_dim) return fail(SWQ_ERR_BAD_SHAPE, "row stride below row size");
    const int splits = swq::attention_splits(rows, num_kv_heads, max_seq, dev.num_sms);
    return launch_status(swq::attention_launch(out, q, k_cache, v_cache, pos, workspace, num_heads, num_kv_heads,
                                               head_dim, rows, max_seq, splits, ldq,
                                               reinterpret_cast<cudaStream_t>(stream)),
                         "attention launch");
}

swq_status swq_silu_mul(float* out, const float* gate, const float* up, int n, int rows, int ld, swq_stream_t stream) {
    if (n < 0 || rows < 0 || ld < n) return fail(SWQ_ERR_BAD_SHAPE, "bad silu_mul sizes");
    if (n == 0 || rows == 0) return SWQ_OK;
    if (!out || !gate || !up) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(
        swq::silu_mul_launch(out, gate, up, n, rows, ld, dev.num_sms, reinterpret_cast<cudaStream_t>(stream)),
        "silu_mul launch");
}

swq_status swq_add(float* x, const float* y, int64_t n, swq_stream_t stream) {
    if (n < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative size");
    if (n == 0) return SWQ_OK;
    if (!x || !y) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::add_launch(x, y, n, dev.num_sms, reinterpret_cast<cudaStream_t>(stream)), "add launch");
}

swq_status swq_embed(float* x, const float* table, const int* tokens, int dim, int vocab, int rows,
                     swq_stream_t stream) {
    if (dim < 0 || rows < 0 || vocab <= 0) return fail(SWQ_ERR_BAD_SHAPE, "bad embedding sizes");
    if (dim == 0 || rows == 0) return SWQ_OK;
    if (!x || !table || !tokens) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::embed_launch(x, table, tokens, dim, vocab, rows, reinterpret_cast<cudaStream_t>(stream)),
                         "embed launch");
}

swq_status swq_argmax(const float* logits, int n, int rows, int* tokens, int* history, const int* step,
                      swq_stream_t stream) {
    if (n <= 0 || rows < 0) return fail(SWQ_ERR_BAD_SHAPE, "bad argmax sizes");
    if (rows == 0) return SWQ_OK;
    if (!logits || !tokens || (history && !step)) return fail(SWQ_ERR_NULL_PTR, "null pointer");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(
        swq::argmax_launch(logits, n, rows, tokens, history, step, reinterpret_cast<cudaStream_t>(stream)),
        "argmax launch");
}

swq_status swq_decode_advance(int* pos, int* step, swq_stream_t stream) {
    if (!pos) return fail(SWQ_ERR_NULL_PTR, "null pos");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::advance_launch(pos, step, reinterpret_cast<cudaStream_t>(stream)), "advance launch");
}

swq_status swq_gemv(int type, const void* W, const float* x, float* y, int N, int K, swq_stream_t stream) {
    return swq_gemm(type, W, x, y, 1, N, K, stream);
}

swq_status swq_check(swq_stream_t stream) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    unsigned a = 0, b = 0, c = 0, d = 0, m = 0, a2 = 0, a3 = 0, a4 = 0;
    if ((e = swq::status_fetch_gemv(&a, s)) != cudaSuccess ||
        (e = swq::status_fetch_gemv_imma(&a2, s)) != cudaSuccess ||
        (e = swq::status_fetch_gemv_kq(&a3, s)) != cudaSuccess ||
        (e = swq::status_fetch_gemv_kqm(&a4, s)) != cudaSuccess ||
        (e = swq::status_fetch_dequant(&b, s)) != cudaSuccess ||
        (e = swq::status_fetch_gemm_tc(&c, s)) != cudaSuccess ||
        (e = swq::status_fetch_allreduce(&d, s)) != cudaSuccess ||
        (e = swq::status_fetch_moe(&m, s)) != cudaSuccess)
        return cuda_fail(e, "status fetch");
    a |= a2 | a3 | a4;
    if (m & swq::kStatusBadId) {
        char buf[128];
        std::snprintf(buf, sizeof(buf), "an expert id outside [0, n_experts) was left out of the MoE sort "
                                        "(status moe=%#x)", m);
        return fail(SWQ_ERR_BAD_ARG, buf);
    }
    d |= m;
    if ((a | b | c | d) & swq::kStatusBadAlign) {
        char buf[160];
        std::snprintf(buf, sizeof(buf),
                      "an expert matrix given to swq_grouped_gemv is not 16-byte aligned; its rows were skipped "
                      "(status gemv=%#x)", a);
        return fail(SWQ_ERR_BAD_ARG, buf);
    }
    if (a | b | c | d) {
        char buf[128];
        std::snprintf(buf, sizeof(buf), "device wait timeout (gemv=%#x dequant=%#x gemm=%#x allreduce=%#x)", a, b,
                      c, d);
        return fail(SWQ_ERR_TIMEOUT, buf);
    }
    return SWQ_OK;
}

// ---------------------------------------------------------------------------
// Peer-memory all-reduce of a tensor-parallel group (one process per GPU).
// ---------------------------------------------------------------------------

static_assert(sizeof(cudaIpcMemHandle_t) == SWQ_ALLREDUCE_HANDLE_BYTES, "IPC handle size");

struct swq_allreduce {
    int device = -1;
    int rank = 0, world = 1;
    size_t max_elems = 0;
    void* own = nullptr;
    void* peer[SWQ_AR_MAX_RANKS] = {};
    swq::ArBuffer bufs[SWQ_AR_MAX_RANKS] = {};
    bool opened = false;
};

swq_status swq_allreduce_create(size_t max_elems, int rank, int world, swq_allreduce** out, void* handle_out) {
    if (!out || !handle_out) return fail(SWQ_ERR_NULL_PTR, "null output pointer");
    *out = nullptr;
    if (world < 1 || world > SWQ_AR_MAX_RANKS || rank < 0 || rank >= world)
        return fail(SWQ_ERR_BAD_ARG, "rank/world outside 0 <= rank < world <= 8");
    if (max_elems == 0) return fail(SWQ_ERR_BAD_SHAPE, "max_elems must be positive");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    auto* ar = new swq_allreduce();
    ar->device = dev.device;
    ar->rank = rank;
    ar->world = world;
    ar->max_elems = max_elems;
    const size_t bytes = swq::allreduce_buffer_bytes(max_elems);
    cudaError_t e = cudaMalloc(&ar->own, bytes);
    if (e == cudaSuccess) e = cudaMemset(ar->own, 0, bytes);  // flags and epochs start at 0
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ar->own);
    if (e != cudaSuccess) {
        if (ar->own) cudaFree(ar->own);
        delete ar;
        return cuda_fail(e, "all-reduce buffer");
    }
    std::memcpy(handle_out, &h, sizeof(h));
    ar->bufs[rank] = swq::ar_view(ar->own, max_elems);
    *out = ar;
    return SWQ_OK;
}

swq_status swq_allreduce_open(swq_allreduce* ar, const void* handles) {
    if (!ar || !handles) return fail(SWQ_ERR_NULL_PTR, "null all-reduce or handles");
    if (ar->opened) return fail(SWQ_ERR_BAD_ARG, "peers already opened");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ar->device) return fail(SWQ_ERR_BAD_ARG, "current device is not the all-reduce's device");
    for (int r = 0; r < ar->world; ++r) {
        if (r == ar->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(r) * SWQ_ALLREDUCE_HANDLE_BYTES,
                    sizeof(h));
        cudaError_t e = cudaIpcOpenMemHandle(&ar->peer[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (ar->peer[q]) {
                    cudaIpcCloseMemHandle(ar->peer[q]);
                    ar->peer[q] = nullptr;
                }
            return cuda_fail(e, "cudaIpcOpenMemHandle");
        }
        ar->bufs[r] = swq::ar_view(ar->peer[r], ar->max_elems);
    }
    ar->opened = true;
    return SWQ_OK;
}

swq_status swq_allreduce_sum(swq_allreduce* ar, float* data, size_t n, swq_stream_t stream) {
    if (!ar || !data) return fail(SWQ_ERR_NULL_PTR, "null all-reduce or data");
    if (!ar->opened && ar->world > 1) return fail(SWQ_ERR_BAD_ARG, "swq_allreduce_open has not run");
    if (n > ar->max_elems) return fail(SWQ_ERR_BAD_SHAPE, "vector longer than the all-reduce buffer");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    if (dev.device != ar->device) return fail(SWQ_ERR_BAD_ARG, "current device is not the all-reduce's device");
    return launch_status(swq::allreduce_launch(ar->bufs, ar->rank, ar->world, data, n, dev.num_sms,
                                               reinterpret_cast<cudaStream_t>(stream)),
                         "all-reduce launch");
}

swq_status swq_allreduce_reset(swq_allreduce* ar, swq_stream_t stream) {
    if (!ar) return fail(SWQ_ERR_NULL_PTR, "null all-reduce");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ar->device) return fail(SWQ_ERR_BAD_ARG, "current device is not the all-reduce's device");
    // Only this rank's own flag words and epoch counters: every rank resets its
    // own, so after the caller's second barrier all ranks count from epoch 0.
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ar->own, 0, swq::ar_header_bytes(), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "all-reduce reset");
}

swq_status swq_allreduce_destroy(swq_allreduce* ar) {
    if (!ar) return SWQ_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(ar->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < ar->world; ++r)
        if (ar->peer[r]) cudaIpcCloseMemHandle(ar->peer[r]);
    if (ar->own) cudaFree(ar->own);
    if (cur >= 0) cudaSetDevice(cur);
    delete ar;
    return SWQ_OK;
}

// ---------------------------------------------------------------------------
// MoE routing, sort and combine; expert-parallel dispatch over peer memory.
// ---------------------------------------------------------------------------

static swq_status moe_shape_check(int T, int E, int k) {
    if (T < 0 || E < 1 || k < 1) return fail(SWQ_ERR_BAD_SHAPE, "need T >= 0, n_experts >= 1, k >= 1");
    if (E > SWQ_MOE_MAX_EXPERTS) return fail(SWQ_ERR_BAD_SHAPE, "more than SWQ_MOE_MAX_EXPERTS experts");
    if (k > SWQ_MOE_MAX_TOPK || k > E) return fail(SWQ_ERR_BAD_SHAPE, "k above SWQ_MOE_MAX_TOPK or n_experts");
    return SWQ_OK;
}

swq_status swq_moe_router(const float* router_w, const float* X, int T, int E, int H, int k, float* logits,
                          int* topk_ids, float* topk_w, swq_stream_t stream) {
    swq_status st = moe_shape_check(T, E, k);
    if (st != SWQ_OK) return st;
    if (H < 1) return fail(SWQ_ERR_BAD_SHAPE, "hidden size must be positive");
    if (T == 0) return SWQ_OK;
    if (!router_w || !X || !logits || !topk_ids || !topk_w) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    if ((st = current_device(&dev)) != SWQ_OK) return st;
    if (static_cast<size_t>(H) * sizeof(float) > static_cast<size_t>(dev.smem_per_block_optin))
        return fail(SWQ_ERR_BAD_SHAPE, "hidden size too large for one token row in shared memory");
    return launch_status(swq::moe_router_launch(router_w, X, logits, T, E, H, k, topk_ids, topk_w,
                                                dev.smem_per_block_optin, reinterpret_cast<cudaStream_t>(stream)),
                         "MoE router launch");
}

swq_status swq_moe_sort(const int* topk_ids, int P, int n_experts, int* expert_offsets, int* sorted_pairs,
                        int* pair_rows, swq_stream_t stream) {
    if (P < 0 || n_experts < 1) return fail(SWQ_ERR_BAD_SHAPE, "need P >= 0 and n_experts >= 1");
    if (n_experts > SWQ_MOE_MAX_EXPERTS) return fail(SWQ_ERR_BAD_SHAPE, "more than SWQ_MOE_MAX_EXPERTS experts");
    if (!expert_offsets || (P > 0 && (!topk_ids || !sorted_pairs || !pair_rows)))
        return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::moe_sort_launch(topk_ids, P, n_experts, expert_offsets, sorted_pairs, pair_rows,
                                              reinterpret_cast<cudaStream_t>(stream)),
                         "MoE sort launch");
}

swq_status swq_moe_gather(const float* X, const int* sorted_pairs, const int* expert_offsets, int n_experts, int P,
                          int k, int H, float* X_sorted, swq_stream_t stream) {
    if (P < 0 || n_experts < 1 || k < 1 || H < 1) return fail(SWQ_ERR_BAD_SHAPE, "bad size");
    if (P == 0) return SWQ_OK;
    if (!X || !sorted_pairs || !expert_offsets || !X_sorted) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::moe_gather_launch(X, sorted_pairs, expert_offsets, n_experts, P, k, H, X_sorted,
                                                dev.num_sms, reinterpret_cast<cudaStream_t>(stream)),
                         "MoE gather launch");
}

swq_status swq_moe_combine(const float* Y_sorted, const int* pair_rows, const float* topk_w, int T, int k, int H,
                           float* Y, int accumulate, swq_stream_t stream) {
    if (T < 0 || k < 1 || H < 1) return fail(SWQ_ERR_BAD_SHAPE, "bad size");
    if (T == 0) return SWQ_OK;
    if (!Y_sorted || !pair_rows || !topk_w || !Y) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    return launch_status(swq::moe_combine_launch(Y_sorted, pair_rows, topk_w, T, k, H, Y, accumulate ? 1 : 0,
                                                 dev.num_sms, reinterpret_cast<cudaStream_t>(stream)),
                         "MoE combine launch");
}

static_assert(sizeof(cudaIpcMemHandle_t) == SWQ_EP_HANDLE_BYTES, "IPC handle size");

struct swq_ep {
    int device = -1;
    int rank = 0;
    swq::EpShape shape{};
    void* own = nullptr;
    void* peer[SWQ_EP_MAX_RANKS] = {};
    swq::EpView bufs[SWQ_EP_MAX_RANKS] = {};
    bool opened = false;
};

swq_status swq_ep_create(int max_tokens, int top_k, int n_experts, int hidden, int rank, int world, swq_ep** out,
                         void* handle_out) {
    if (!out || !handle_out) return fail(SWQ_ERR_NULL_PTR, "null output pointer");
    *out = nullptr;
    if (world < 1 || world > SWQ_EP_MAX_RANKS || rank < 0 || rank >= world)
        return fail(SWQ_ERR_BAD_ARG, "rank/world outside 0 <= rank < world <= SWQ_EP_MAX_RANKS");
    swq_status st = moe_shape_check(max_tokens, n_experts, top_k);
    if (st != SWQ_OK) return st;
    if (max_tokens < 1 || hidden < 1) return fail(SWQ_ERR_BAD_SHAPE, "max_tokens and hidden must be positive");
    if (n_experts % world) return fail(SWQ_ERR_BAD_SHAPE, "n_experts must split evenly over the ranks");
    if (static_cast<int64_t>(max_tokens) * top_k * world > (1 << 30))
        return fail(SWQ_ERR_BAD_SHAPE, "max_tokens * top_k * world above 2^30 rows");
    swq::DeviceInfo dev;
    if ((st = current_device(&dev)) != SWQ_OK) return st;
    auto* ep = new swq_ep();
    ep->device = dev.device;
    ep->rank = rank;
    ep->shape = swq::EpShape{max_tokens, top_k, n_experts, hidden, world};
    const size_t bytes = swq::ep_buffer_bytes(ep->shape);
    cudaError_t e = cudaMalloc(&ep->own, bytes);
    if (e == cudaSuccess) e = cudaMemset(ep->own, 0, swq::ep_header_bytes());  // flags, epoch, meta start at 0
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ep->own);
    if (e != cudaSuccess) {
        if (ep->own) cudaFree(ep->own);
        delete ep;
        return cuda_fail(e, "expert-parallel buffer");
    }
    std::memcpy(handle_out, &h, sizeof(h));
    ep->bufs[rank] = swq::ep_view(ep->own, ep->shape);
    if (world == 1) ep->opened = true;
    *out = ep;
    return SWQ_OK;
}

swq_status swq_ep_open(swq_ep* ep, const void* handles) {
    if (!ep || !handles) return fail(SWQ_ERR_NULL_PTR, "null expert-parallel object or handles");
    if (ep->opened && ep->shape.world > 1) return fail(SWQ_ERR_BAD_ARG, "peers already opened");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ep->device) return fail(SWQ_ERR_BAD_ARG, "current device is not the expert-parallel object's device");
    for (int r = 0; r < ep->shape.world; ++r) {
        if (r == ep->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(r) * SWQ_EP_HANDLE_BYTES,
                    sizeof(h));
        cudaError_t e = cudaIpcOpenMemHandle(&ep->peer[r], h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (ep->peer[q]) {
                    cudaIpcCloseMemHandle(ep->peer[q]);
                    ep->peer[q] = nullptr;
                }
            return cuda_fail(e, "cudaIpcOpenMemHandle");
        }
        ep->bufs[r] = swq::ep_view(ep->peer[r], ep->shape);
    }
    ep->opened = true;
    return SWQ_OK;
}

static swq_status ep_ready(const swq_ep* ep) {
    if (!ep) return fail(SWQ_ERR_NULL_PTR, "null expert-parallel object");
    if (!ep->opened) return fail(SWQ_ERR_BAD_ARG, "swq_ep_open has not run");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ep->device) return fail(SWQ_ERR_BAD_ARG, "current device is not the expert-parallel object's device");
    return SWQ_OK;
}

swq_status swq_ep_dispatch(swq_ep* ep, const float* X, const int* topk_ids, int T, swq_stream_t stream) {
    swq_status st = ep_ready(ep);
    if (st != SWQ_OK) return st;
    if (T < 0 || T > ep->shape.max_tokens) return fail(SWQ_ERR_BAD_SHAPE, "T outside 0 .. max_tokens");
    if (T > 0 && (!X || !topk_ids)) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    return launch_status(swq::ep_dispatch_launch(ep->bufs, ep->rank, ep->shape, topk_ids, X, T,
                                                 reinterpret_cast<cudaStream_t>(stream)),
                         "expert-parallel dispatch launch");
}

swq_status swq_ep_received(const swq_ep* ep, float** X_recv, const int** expert_offsets, int* capacity) {
    if (!ep || !X_recv || !expert_offsets || !capacity) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    *X_recv = ep->bufs[ep->rank].rbuf;
    *expert_offsets = ep->bufs[ep->rank].loff;
    *capacity = ep->shape.max_tokens * ep->shape.k * ep->shape.world;
    return SWQ_OK;
}

swq_status swq_ep_combine(swq_ep* ep, const float* Y_recv, const float* topk_w, float* Y, int accumulate,
                          swq_stream_t stream) {
    swq_status st = ep_ready(ep);
    if (st != SWQ_OK) return st;
    if (!Y_recv || !topk_w || !Y) return fail(SWQ_ERR_NULL_PTR, "null pointer argument");
    return launch_status(swq::ep_combine_launch(ep->bufs, ep->rank, ep->shape, Y_recv, topk_w, Y,
                                                accumulate ? 1 : 0, reinterpret_cast<cudaStream_t>(stream)),
                         "expert-parallel combine launch");
}

swq_status swq_ep_reset(swq_ep* ep, swq_stream_t stream) {
    if (!ep) return fail(SWQ_ERR_NULL_PTR, "null expert-parallel object");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != ep->device) return fail(SWQ_ERR_BAD_ARG, "current device is not the expert-parallel object's device");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(ep->own, 0, swq::ep_header_bytes(), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? SWQ_OK : cuda_fail(e, "expert-parallel reset");
}

swq_status swq_ep_destroy(swq_ep* ep) {
    if (!ep) return SWQ_OK;
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(ep->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < ep->shape.world; ++r)
        if (ep->peer[r]) cudaIpcCloseMemHandle(ep->peer[r]);
    if (ep->own) cudaFree(ep->own);
    if (cur >= 0) cudaSetDevice(cur);
    delete ep;
    return SWQ_OK;
}

// ---------------------------------------------------------------------------
// Host-buffer context: the reference's calling convention.
// ---------------------------------------------------------------------------

struct swq_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    struct Entry {
        void* dev = nullptr;
        size_t bytes = 0;
        int type = 0, N = 0, K = 0;
    };
    std::map<const void*, std::vector<Entry>> cache;
    size_t resident = 0;
    // device activation/output buffers and pinned staging, grown on demand
    float* d_x = nullptr;
    float* d_y = nullptr;
    size_t cap_x = 0, cap_y = 0;
    float* h_x = nullptr;
    float* h_y = nullptr;
    size_t hcap_x = 0, hcap_y = 0;
};

namespace {

swq_status ensure_dev(float** p, size_t* cap, size_t need) {
    if (*cap >= need) return SWQ_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), need);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    *cap = need;
    return SWQ_OK;
}

swq_status ensure_host(float** p, size_t* cap, size_t need) {
    if (*cap >= need) return SWQ_OK;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    cudaError_t e = cudaMallocHost(reinterpret_cast<void**>(p), need);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMallocHost");
    *cap = need;
    return SWQ_OK;
}

swq_status resident_weight(swq_ctx* c, const void* w, int type, int N, int K, size_t bytes, const void** dev) {
    auto& v = c->cache[w];
    for (auto& en : v) {
        if (en.type == type && en.N == N && en.K == K) {
            *dev = en.dev;
            return SWQ_OK;
        }
    }
    swq_ctx::Entry en;
    cudaError_t e = cudaMalloc(&en.dev, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(weights)");
    e = cudaMemcpy(en.dev, w, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(en.dev);
        return cuda_fail(e, "cudaMemcpy(weights)");
    }
    en.bytes = bytes;
    en.type = type;
    en.N = N;
    en.K = K;
    v.push_back(en);
    c->resident += bytes;
    *dev = en.dev;
    return SWQ_OK;
}

}  // namespace

swq_status swq_ctx_create(int device, swq_ctx_t* out) {
    if (!out) return fail(SWQ_ERR_NULL_PTR, "null ctx out");
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    swq::DeviceInfo dev;
    swq_status st = current_device(&dev);
    if (st != SWQ_OK) return st;
    auto* c = new swq_ctx();
    c->device = device;
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaStreamCreate");
    }
    *out = c;
    return SWQ_OK;
}

swq_status swq_ctx_destroy(swq_ctx_t c) {
    if (!c) return SWQ_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto& kv : c->cache)
        for (auto& en : kv.second) cudaFree(en.dev);
    if (c->d_x) cudaFree(c->d_x);
    if (c->d_y) cudaFree(c->d_y);
    if (c->h_x) cudaFreeHost(c->h_x);
    if (c->h_y) cudaFreeHost(c->h_y);
    cudaStreamDestroy(c->stream);
    delete c;
    return SWQ_OK;
}

swq_status swq_ctx_matmul_q_batched(swq_ctx_t c, float* Y, const float* X, const void* w, int type, int M, int N,
                                    int K) {
    if (!c) return fail(SWQ_ERR_NULL_PTR, "null ctx");
    TypeInfo ti;
    swq_status st = check_gemm_args(type, w, X, Y, M, N, K, &ti);
    if (st != SWQ_OK || M == 0 || N == 0) return st;
    std::lock_guard<std::mutex> lk(c->mu);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    const size_t wbytes = static_cast<size_t>(N) * (K / ti.qk) * ti.bb;
    const void* dW = nullptr;
    if (K > 0 && (st = resident_weight(c, w, type, N, K, wbytes, &dW)) != SWQ_OK) return st;
    const size_t xb = sizeof(float) * static_cast<size_t>(M) * K, yb = sizeof(float) * static_cast<size_t>(M) * N;
    if ((st = ensure_dev(&c->d_x, &c->cap_x, std::max<size_t>(xb, 16))) != SWQ_OK ||
        (st = ensure_dev(&c->d_y, &c->cap_y, yb)) != SWQ_OK ||
        (st = ensure_host(&c->h_x, &c->hcap_x, std::max<size_t>(xb, 16))) != SWQ_OK ||
        (st = ensure_host(&c->h_y, &c->hcap_y, yb)) != SWQ_OK)
        return st;
    if (xb) std::memcpy(c->h_x, X, xb);
    if (xb && (e = cudaMemcpyAsync(c->d_x, c->h_x, xb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return cuda_fail(e, "H2D x");
    st = swq_gemm(type, dW ? dW : c->d_x, c->d_x, c->d_y, M, N, K, reinterpret_cast<swq_stream_t>(c->stream));
    if (st != SWQ_OK) return st;
    if ((e = cudaMemcpyAsync(c->h_y, c->d_y, yb, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return cuda_fail(e, "D2H y");
    if ((e = cudaStreamSynchronize(c->stream)) != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    std::memcpy(Y, c->h_y, yb);
    return SWQ_OK;
}

swq_status swq_ctx_matmul_transposed_q(swq_ctx_t c, float* out, const float* x, const void* w, int type, int N,
                                       int K) {
    return swq_ctx_matmul_q_batched(c, out, x, w, type, 1, N, K);
}

swq_status swq_ctx_dequantize(swq_ctx_t c, const void* src, float* dst, int64_t n, int type) {
    if (!c) return fail(SWQ_ERR_NULL_PTR, "null ctx");
    TypeInfo ti;
    if (!type_info(type, &ti)) return fail(SWQ_ERR_BAD_TYPE, "type " + std::to_string(type) + " is not on this path");
    if (n < 0) return fail(SWQ_ERR_BAD_SHAPE, "negative n");
    const int64_t nblocks = n / ti.qk;
    if (nblocks == 0) return SWQ_OK;
    if (!src || !dst) return fail(SWQ_ERR_NULL_PTR, "null src or dst");
    std::lock_guard<std::mutex> lk(c->mu);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    const size_t inb = static_cast<size_t>(nblocks) * ti.bb;
    const size_t outb = sizeof(float) * static_cast<size_t>(nblocks) * ti.qk;
    void* d_in = nullptr;
    float* d_out = nullptr;
    if ((e = cudaMalloc(&d_in, inb)) != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    if ((e = cudaMalloc(reinterpret_cast<void**>(&d_out), outb)) != cudaSuccess) {
        cudaFree(d_in);
        return cuda_fail(e, "cudaMalloc");
    }
    swq_status st = SWQ_OK;
    if ((e = cudaMemcpyAsync(d_in, src, inb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        st = cuda_fail(e, "H2D blocks");
    if (st == SWQ_OK) st = swq_dequant(type, d_in, d_out, n, reinterpret_cast<swq_stream_t>(c->stream));
    if (st == SWQ_OK && (e = cudaMemcpyAsync(dst, d_out, outb, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        st = cuda_fail(e, "D2H out");
    if (st == SWQ_OK && (e = cudaStreamSynchronize(c->stream)) != cudaSuccess) st = cuda_fail(e, "sync");
    cudaFree(d_in);
    cudaFree(d_out);
    return st;
}

swq_status swq_ctx_evict(swq_ctx_t c, const void* w) {
    if (!c) return fail(SWQ_ERR_NULL_PTR, "null ctx");
    std::lock_guard<std::mutex> lk(c->mu);
    auto it = c->cache.find(w);
    if (it == c->cache.end()) return SWQ_OK;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto& en : it->second) {
        cudaFree(en.dev);
        c->resident -= en.bytes;
    }
    c->cache.erase(it);
    return SWQ_OK;
}

size_t swq_ctx_resident_bytes(swq_ctx_t c) { return c ? c->resident : 0; }

}  // extern "C"
