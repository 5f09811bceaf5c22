// moe.h -- internal interface of the MoE routing / sort / combine kernels and
// of the expert-parallel dispatch over peer memory (host side).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "../../include/swq.h"

namespace swq {

// Status bit of an expert id out of range (DEV_BAD_ID in the device word).
constexpr unsigned kStatusBadId = 64u;
enum { EP_CTAS = 128 };  // CTAs of the dispatch and combine kernels (flag slots per rank)
enum { EP_META_OK = 0, EP_META_P = 1, EP_META_T = 2, EP_META_ROWS = 3, EP_META_WORDS = 8 };

// One rank's expert-parallel buffer as mapped in this process.  The header
// (flags, epoch, meta) comes first: zeroing it resets the rank.
struct EpView {
    unsigned* cflag;  // [MAX_RANKS]            count matrix row s published (epoch)
    unsigned* dflag;  // [MAX_RANKS][EP_CTAS]   rows of source s, CTA b, arrived
    unsigned* rflag;  // [MAX_RANKS][EP_CTAS]   outputs returned by rank d, CTA b
    unsigned* epoch;  // [1]                    this rank's call counter
    int* meta;        // [EP_META_WORDS]        ok, pairs, tokens, rows of the call
    int* cm;          // [MAX_RANKS][E]         per-expert pair counts of every source
    int* loff;        // [E/world + 1]          this rank's experts' row offsets
    int* spair;       // [max_tokens * k]       my pairs sorted by expert
    int* prow;        // [max_tokens * k]       sorted slot of each pair (-1: bad id)
    int* drow;        // [max_tokens * k]       destination row of each sorted slot
    int2* rtag;       // [cap]                  (source, slot) of each received row
    float* rbuf;      // [cap][H]               received rows, by local expert
    float* ret;       // [max_tokens * k][H]    expert outputs of my sorted slots
};

struct EpShape {
    int max_tokens, k, E, H, world;
};

size_t ep_header_bytes();
size_t ep_buffer_bytes(const EpShape& sh);
EpView ep_view(void* base, const EpShape& sh);

// Router GEMV (fp32) into logits [T][E], then top-k + softmax into ids/w [T][k].
cudaError_t moe_router_launch(const float* Wr, const float* X, float* logits, int T, int E, int H, int k, int* ids,
                              float* w, int smem_max, cudaStream_t s);
cudaError_t moe_sort_launch(const int* ids, int P, int E, int* offsets, int* sorted, int* prow, cudaStream_t s);
cudaError_t moe_gather_launch(const float* X, const int* sorted, const int* offsets, int E, int P, int k, int H,
                              float* Xs, int num_sms, cudaStream_t s);
cudaError_t moe_combine_launch(const float* Ys, const int* prow, const float* w, int T, int k, int H, float* Y,
                               int accumulate, int num_sms, cudaStream_t s);
// Route (one CTA) + dispatch (EP_CTAS CTAs) of T tokens' top-k pairs.
cudaError_t ep_dispatch_launch(const EpView* bufs, int rank, const EpShape& sh, const int* ids, const float* X, int T,
                               cudaStream_t s);
cudaError_t ep_combine_launch(const EpView* bufs, int rank, const EpShape& sh, const float* Yr, const float* w,
                              float* Y, int accumulate, cudaStream_t s);
cudaError_t status_fetch_moe(unsigned* out, cudaStream_t s);

}  // namespace swq
