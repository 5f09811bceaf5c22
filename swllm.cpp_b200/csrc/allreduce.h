// allreduce.h -- internal interface of the peer-memory all-reduce (host side).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#define SWQ_AR_MAX_RANKS 8
#define SWQ_AR_MAX_CTAS 256

namespace swq {

// One rank's buffer as mapped in this process: flag words (one per CTA slot,
// written by the owner, read by the peers), the owner's epoch counters, and
// two data halves of half_elems floats.
struct ArBuffer {
    unsigned* flag;
    unsigned* epoch;
    float* data;
    size_t half_elems;
};

size_t ar_header_bytes();
size_t allreduce_buffer_bytes(size_t max_elems);
ArBuffer ar_view(void* base, size_t max_elems);
// Sum `n` floats at `data` over the `world` ranks whose buffers are `bufs`
// (bufs[rank] is this rank's own), in place; every rank makes the same call.
cudaError_t allreduce_launch(const ArBuffer* bufs, int rank, int world, float* data, size_t n, int num_sms,
                             cudaStream_t s);
cudaError_t status_fetch_allreduce(unsigned* out, cudaStream_t s);

}  // namespace swq
