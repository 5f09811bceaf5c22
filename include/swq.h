/*
 * swq.h -- C ABI of libswq, the sm_100a (B200) implementation of swllm.cpp's
 * quantized-weight matmul path: GGUF block dequantization fused into GEMV
 * (decode) and GEMM (prefill), for Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K.
 *
 * Plain C: pointers, sizes and a stream handle.  Device pointers are CUDA
 * device (or managed) memory; every call is asynchronous on `stream` and
 * returns once the work is enqueued.  The caller owns every buffer.  Weights
 * are the GGUF blocks exactly as stored in the file (src/gguf.h:60-118 sizes,
 * src/tensor.h:136-432 layouts): a matrix W[N x K] is N rows of K/QK
 * consecutive blocks, GGUF dims[0] = K, dims[1] = N (src/model.h:729-758).
 *
 * Type ids are the GGMLType values of src/gguf.h:18-40.
 *
 * Numerics (checked by the tests against the reference's own CPU code):
 *   - swq_dequant is bit-exact with the reference's dequantize().
 *   - swq_gemv / swq_gemm are within 1e-3 relative L2 of the reference's
 *     fp32 result on the same inputs.
 */
#ifndef SWQ_H
#define SWQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* swq_stream_t;

typedef enum swq_status {
    SWQ_OK = 0,
    SWQ_ERR_BAD_TYPE = 1,    /* type id not on this path */
    SWQ_ERR_BAD_SHAPE = 2,   /* K % QK != 0, negative sizes, size limits */
    SWQ_ERR_NULL_PTR = 3,    /* a required pointer is NULL */
    SWQ_ERR_CUDA = 4,        /* a CUDA runtime call failed (see swq_last_error) */
    SWQ_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up */
    SWQ_ERR_UNSUPPORTED = 6, /* no sm_100 device, or option value not supported */
    SWQ_ERR_BAD_ARG = 7      /* any other invalid argument */
} swq_status;

/* GGMLType ids on this path (src/gguf.h:18-40). */
enum {
    SWQ_TYPE_Q4_0 = 2,
    SWQ_TYPE_Q8_0 = 8,
    SWQ_TYPE_Q2_K = 10,
    SWQ_TYPE_Q3_K = 11,
    SWQ_TYPE_Q4_K = 12,
    SWQ_TYPE_Q5_K = 13,
    SWQ_TYPE_Q6_K = 14
};

/* Human-readable name of a status code (static storage). */
const char* swq_status_string(swq_status s);

/* Detail of the last error raised on the calling host thread ("" if none). */
const char* swq_last_error(void);

/* Bytes per block and elements per block.  Replaces ggml_type_size /
 * ggml_block_size (src/gguf.h:60-118) for the types on this path; 0 for any
 * other type. */
size_t swq_type_size(int ggml_type);
size_t swq_block_size(int ggml_type);

/* Dequantize n elements of GGUF blocks to fp32, bit-exact with the reference.
 * Replaces dequantize(const void* src, float* dst, int64_t n, GGMLType)
 * (src/tensor.h:451).  As there, n / QK whole blocks are written and a tail of
 * n % QK elements is left untouched; n == 0 is a no-op. */
swq_status swq_dequant(int ggml_type, const void* blocks, float* out, int64_t n,
                       swq_stream_t stream);

/* y[N] = W[N x K] . x[K], fp32 in and out.  Replaces the per-type CPU branch
 * and the host-dequantize CUDA branch of Compute::matmul_transposed_q
 * (src/tensor.h:1212-1278) with one fused kernel on device-resident blocks.
 * K must be a multiple of the block size (32 or 256). */
swq_status swq_gemv(int ggml_type, const void* W, const float* x, float* y,
                    int N, int K, swq_stream_t stream);

/* Y[M x N] = X[M x K] . W[N x K]^T, row-major fp32 X and Y.  The reference has
 * no batched quantized path: its prefill calls Compute::matmul_transposed_q
 * once per token (src/main.cpp:284-287), so this equals M such calls.  Small
 * M runs the fused GEMV kernel; larger M the tensor-core GEMM. */
swq_status swq_gemm(int ggml_type, const void* W, const float* X, float* Y,
                    int M, int N, int K, swq_stream_t stream);

/* ---- Decode step around the GEMVs ------------------------------------------
 *
 * Device-resident forms of the Compute helpers Model::forward calls between
 * its projections (src/model.h:257-543; helpers src/tensor.h:1028-1180,
 * 1280-1340), fp32 as there.  `rows` sequences decode together at the same
 * position, read from device memory (*pos) so a captured step replays for
 * every token.  KV caches are per layer [rows][max_seq][kv_dim] fp32. */

/* out[r] = x[r] / sqrt(mean(x[r]^2) + eps) * w  (Compute::rmsnorm, :1280) */
swq_status swq_rmsnorm(float* out, const float* x, const float* w, int n, float eps, int rows,
                       swq_stream_t stream);
/* x[r] += y[r], then out[r] = rmsnorm(x[r]): a residual add and the RMSNorm
 * that follows it (src/model.h:363-366 then :519-520), in one pass. */
swq_status swq_add_rmsnorm(float* out, float* x, const float* y, const float* w, int n, float eps, int rows,
                           swq_stream_t stream);
/* RoPE of q (in place) and k at position *pos, then k and v into the caches
 * (Compute::rope, :1313, and the cache stores of src/model.h:326-327); freqs
 * [rope_dim/2] = 1/theta^(2i/rope_dim); neox != 0 rotates (i, i + rope_dim/2)
 * pairs, else (2i, 2i+1).  Row r of q, k, v starts at r*ldq, r*ldk, r*ldv
 * (0: q_dim, kv_dim, kv_dim), so q and k may be slices of one projection. */
swq_status swq_rope_kv(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                       const int* pos, const float* freqs, int q_dim, int kv_dim, int head_dim,
                       int rope_dim, int neox, int rows, int max_seq, int ldq, int ldk, int ldv,
                       swq_stream_t stream);
/* The optional steps between the q/k/v projections and RoPE of the reference's
 * dense forward (src/model.h:291-318): q += bq, k += bk, v += bv
 * (Compute::add), then the RMSNorm of every q head with q_norm and every k
 * head with k_norm ([head_dim] weights shared by the heads; Compute::rmsnorm
 * with rms_norm_eps).  In place on `rows` rows (strides ldq / ldk / ldv, 0:
 * packed); any of the six vectors may be NULL (nothing to do for it). */
swq_status swq_qkv_bias_norm(float* q, float* k, float* v, const float* bq, const float* bk, const float* bv,
                              const float* q_norm, const float* k_norm, int q_dim, int kv_dim, int head_dim,
                              float eps, int rows, int ldq, int ldk, int ldv, swq_stream_t stream);
/* One decode step of a GatedDeltaNet (linear attention) layer after its
 * projections: the reference's Qwen3.5 branch of Model::forward from the
 * q/k/v, gate, beta, alpha and dt projections to the input of the output
 * projection (src/model.h:421-504).  Per row r:
 *   v = causal depthwise conv1d of the value channels over conv_width steps
 *       (the history conv_state[r][d][0..conv_width) shifts left, v enters
 *       last; conv_w [value_dim][conv_width]; NULL conv_w: v unchanged);
 *   per value head h (key head h mod n_k_heads, k_hd = key_head_dim,
 *   v_hd = value_head_dim): decay = exp(-exp(ssm_a[h]) * sigmoid(alpha[h])
 *   * sigmoid(dt[h])), beta = sigmoid(beta[h]) (NULL alpha / dt / ssm_a /
 *   beta: the factor is 1); pred = S^T k; S = decay S + beta k (v - pred)^T;
 *   y = S^T q with S = state[r][h] [k_hd][v_hd];
 *   y = rmsnorm(y over the head, eps 1e-5) * norm_w (NULL: no norm);
 *   y *= sigmoid(z) (NULL z: sigmoid(0), as the reference gates without the
 *   projection).
 * qkv rows (stride ld_qkv, 0: packed) hold q [n_k*k_hd], k [n_k*k_hd],
 * v [n_v*v_hd]; z [rows][n_v*v_hd]; beta, alpha, dt [rows][n_v]; y
 * [rows][n_v*v_hd].  The state and conv history are updated in place (zero
 * them to start a sequence).  value_head_dim <= 1024. */
swq_status swq_gdn_step(const float* qkv, int ld_qkv, const float* z, const float* beta, const float* alpha,
                        const float* dt, const float* ssm_a, const float* conv_w, const float* norm_w, float* state,
                        float* conv_state, float* y, int rows, int n_k_heads, int n_v_heads, int key_head_dim,
                        int value_head_dim, int conv_width, swq_stream_t stream);
/* Prefill: no counterpart in the reference, which runs a prompt as one
 * Model::forward per token (src/main.cpp:284-287).  The prompt's seq_len
 * tokens of num_seqs sequences are the rows m = s*seq_len + p of q / k / v /
 * out (token p of sequence s, at position pos0 + p; pos0 + seq_len <= max_seq),
 * so the projections around these calls are M-row swq_gemm calls.
 * swq_rope_kv_prefill: swq_rope_kv at each row's own position, k and v into
 * the cache of the row's sequence.  swq_attention_prefill: causal
 * grouped-query attention, row m over positions 0 .. pos0 + p of its
 * sequence (src/model.h:329-361); allocates nothing; head_dim 32/64/128/256.
 * Strides 0 mean packed rows. */
swq_status swq_rope_kv_prefill(float* q, const float* k, const float* v, float* k_cache, float* v_cache,
                               int pos0, int seq_len, const float* freqs, int q_dim, int kv_dim, int head_dim,
                               int rope_dim, int neox, int num_seqs, int max_seq, int ldq, int ldk, int ldv,
                               swq_stream_t stream);
swq_status swq_attention_prefill(float* out, const float* q, const float* k_cache, const float* v_cache,
                                 int pos0, int seq_len, int num_heads, int num_kv_heads, int head_dim,
                                 int num_seqs, int max_seq, int ldq, int ldo, swq_stream_t stream);
/* Grouped-query decode attention over positions 0 .. *pos (src/model.h:329-361),
 * split over the context; the last split of each (sequence, kv head) merges
 * the others.  `workspace`: swq_attention_workspace_bytes() bytes, caller-owned
 * (the call allocates nothing), zero-filled before its first use; every call
 * leaves it zeroed again.  Row r of q starts at r*ldq (0: num_heads*head_dim).
 * out is rows x num_heads*head_dim. */
size_t swq_attention_workspace_bytes(int num_heads, int num_kv_heads, int head_dim, int rows, int max_seq);
swq_status swq_attention_decode(float* out, const float* q, const float* k_cache, const float* v_cache,
                                const int* pos, void* workspace, size_t workspace_bytes, int num_heads,
                                int num_kv_heads, int head_dim, int rows, int max_seq, int ldq,
                                swq_stream_t stream);
/* out[r][i] = silu(gate[r*ld + i]) * up[r*ld + i]  (Compute::silu_mul, :1300) */
swq_status swq_silu_mul(float* out, const float* gate, const float* up, int n, int rows, int ld,
                        swq_stream_t stream);
/* x += y  (Compute::add, :1336) */
swq_status swq_add(float* x, const float* y, int64_t n, swq_stream_t stream);
/* x[r] = table[tokens[r]], fp32 rows of `dim` (src/model.h:265); a token id
 * outside [0, vocab) reads row 0. */
swq_status swq_embed(float* x, const float* table, const int* tokens, int dim, int vocab, int rows,
                     swq_stream_t stream);
/* tokens[r] = argmax of logits[r] (first maximum; 0 when no element exceeds
 * -inf, e.g. all NaN); history[*step * rows + r] too when history is not NULL
 * (greedy sampling). */
swq_status swq_argmax(const float* logits, int n, int rows, int* tokens, int* history, const int* step,
                      swq_stream_t stream);
/* *pos += 1 and, when step is not NULL, *step += 1 */
swq_status swq_decode_advance(int* pos, int* step, swq_stream_t stream);

/* ---- MoE grouped expert GEMM ---------------------------------------------
 *
 * For each expert e: Y[r] = X[r] . W_e^T for the rows r = expert_offsets[e] ..
 * expert_offsets[e+1]-1, i.e. the expert FFN projections of a mixture-of-experts
 * layer after the tokens (or token x top-k slots) have been grouped by expert.
 * The reference has no MoE path (its FFN is dense, src/model.h:520-528; the
 * GGUF expert tensor names only appear at src/hf_loader.h:474-493), so this
 * replaces the per-expert loop of Compute::matmul_transposed_q calls
 * (src/tensor.h:1212) a MoE forward would make.
 *   W_experts       device array of n_experts device pointers, each to an
 *                   N x K GGUF matrix of `ggml_type` (any alignment)
 *   expert_offsets  device int array of n_experts + 1 row offsets into X/Y;
 *                   entries are clamped to [0, total_rows] and a decreasing
 *                   step is read as an empty expert
 *   X_sorted, Y     device fp32, total_rows x K and total_rows x N, row-major
 * Rows outside every expert's range are left untouched.  Runs the tensor-core
 * GEMM (fp16 operands, fp32 accumulation; same tolerance as swq_gemm) with a
 * temporary fp16 copy of X from libswq's stream-ordered pool.  n_experts <=
 * 4095. */
swq_status swq_grouped_gemm(int ggml_type, const void* const* W_experts, const int* expert_offsets,
                            const float* X_sorted, float* Y, int n_experts, int total_rows,
                            int N, int K, swq_stream_t stream);

/* ---- Grouped expert matmul for a known expected load ---------------------
 *
 * No counterpart in the reference (no MoE path).  swq_grouped_gemm /
 * swq_grouped_gemv with the kernel picked from mean_rows, the expected rows
 * per expert (for a MoE layer T * k / n_experts, known on the host before the
 * routing runs on the device), where total_rows only bounds the rows (e.g. the
 * capacity that swq_ep_received reports):
 *   mean_rows <= 4: the grouped GEMV (expert matrices 16-byte aligned), each
 *     expert's rows taken in passes of 4, 2 or 1 by its own row count, read
 *     on the device;
 *   else: the tensor-core grouped GEMM with its token tile from mean_rows;
 *     rows of X at or past expert_offsets[n_experts] are not read.
 * expert_offsets must be non-decreasing (as swq_moe_sort and swq_ep_received
 * give them).  A row's result does not depend on the other rows.
 * n_experts <= 4095. */
swq_status swq_grouped_matmul(int ggml_type, const void* const* W_experts, const int* expert_offsets,
                              const float* X_sorted, float* Y, int n_experts, int total_rows, int N, int K,
                              int mean_rows, swq_stream_t stream);
/* swq_grouped_matmul with the experts stacked in one tensor, the layout of a
 * GGUF expert tensor (ffn_{gate,up,down}_exps, [n_experts][N][K] blocks):
 * expert e's matrix is rows e*N .. e*N+N-1 of the n_experts*N x K matrix at
 * W_all.  The tensor-core form then loads each weight stage with one
 * tensor-map copy (W_all 16-byte aligned and row bytes a multiple of 16; else
 * one copy per row). */
swq_status swq_grouped_matmul_stacked(int ggml_type, const void* W_all, const int* expert_offsets,
                                      const float* X_sorted, float* Y, int n_experts, int total_rows, int N, int K,
                                      int mean_rows, swq_stream_t stream);

/* ---- GEMM with a fused activation prologue --------------------------------
 *
 * No counterpart in the reference: its decode step runs RMSNorm
 * (src/tensor.h:1028-1033) and SiLU-mul (src/tensor.h:1050-1064) as separate
 * passes before the projections that read them (src/model.h:272-289,
 * 519-541).  swq_gemm_act computes swq_gemm on a transformed X, the transform
 * done while the kernel stages the activations (no extra pass over memory):
 *   SWQ_ACT_NONE     X as given.
 *   SWQ_ACT_RMSNORM  x = X[m] (+ residual[m] when residual != NULL), then
 *                    x / sqrt(mean(x^2) + eps) * norm_w (K weights).  With
 *                    sum_out != NULL, x (the residual sum) is also written
 *                    there (M x K); sum_out must not overlap X or residual.
 *   SWQ_ACT_SWIGLU   x[k] = silu(g[k]) * u[k] with g = X[m*ld + k] and
 *                    u = X[m*ld + K + k] (gate then up in one row of stride
 *                    ld >= 2K; ld = 0 means 2K).
 * flags: SWQ_GEMM_NOALLOC runs as swq_gemm_noalloc (same limit).  act = NULL
 * is SWQ_ACT_NONE.  Tolerance as swq_gemm (the scale 1/rms is applied to the
 * outputs, in fp32). */
enum { SWQ_ACT_NONE = 0, SWQ_ACT_RMSNORM = 1, SWQ_ACT_SWIGLU = 2 };
enum { SWQ_GEMM_NOALLOC = 1 };
typedef struct swq_act {
    int kind;
    const float* residual;
    const float* norm_w;
    float eps;
    float* sum_out;
    int ld;
} swq_act;
swq_status swq_gemm_act(int ggml_type, const void* W, const float* X, float* Y, int M, int N, int K,
                        const swq_act* act, int flags, swq_stream_t stream);

/* swq_gemm_act with the tensor-core path's scratch (the fp16 copy of X, its
 * row scales, split-K counters and partial products) in a caller-owned
 * workspace instead of libswq's pool.  No counterpart in the reference.  Each
 * owner of a workspace (e.g. each decoder of a process) gets scratch of its
 * own, so calls on different workspaces never share memory; calls on one
 * workspace must not overlap on the GPU.  A call captured in a CUDA graph
 * allocates nothing.
 *   swq_gemm_workspace_bytes: bytes a call of this shape needs on the current
 *     device (0 when it runs the GEMV kernel, which needs none; 0 for
 *     invalid arguments).
 *   workspace: 256-byte aligned; NULL or too small for a call that needs it
 *     is SWQ_ERR_NULL_PTR / SWQ_ERR_BAD_ARG before any device work.  The
 *     counters in it are reset by the call itself: no clearing needed. */
size_t swq_gemm_workspace_bytes(int ggml_type, int M, int N, int K);
swq_status swq_gemm_act_ws(int ggml_type, const void* W, const float* X, float* Y, int M, int N, int K,
                           const swq_act* act, void* workspace, size_t workspace_bytes, swq_stream_t stream);

/* ---- Grouped GEMV for MoE decode ------------------------------------------
 *
 * No counterpart in the reference (it has no MoE path, src/model.h:520-528).
 * The same contract as swq_grouped_gemm, for the decode case of a few rows per
 * expert: a GEMV over each expert's own rows (fixed-point activations, the
 * same tolerance as swq_gemv) instead of the tensor-core GEMM, which works in
 * tiles of 64 or more rows.  Only experts that have rows are read.  Unlike
 * swq_grouped_gemm, every expert matrix must start on a 16-byte boundary; an
 * expert that does not is skipped and swq_check then returns SWQ_ERR_BAD_ARG.
 * Rows per expert are served in groups of 1, 2 or 4 (by the mean of
 * total_rows / n_experts); any count is correct, many rows per expert are
 * faster through swq_grouped_gemm.  n_experts <= 65535. */
swq_status swq_grouped_gemv(int ggml_type, const void* const* W_experts, const int* expert_offsets,
                            const float* X_sorted, float* Y, int n_experts, int total_rows, int N, int K,
                            swq_stream_t stream);

/* ---- Allocation-free GEMM ------------------------------------------------
 *
 * No counterpart in the reference.  swq_gemm's tensor-core path takes a
 * temporary fp16 copy of X (M * K * 2 bytes, plus M fp32 row scales and, for
 * calls with fewer output tiles than half the SMs, split-K partial products)
 * from a stream-ordered memory pool that libswq creates per device and keeps
 * until exit.  Some callers cannot let a library allocate device memory: processes
 * whose own allocator already owns the GPU's memory (a serving engine that
 * reserves what HBM is left for its KV cache at start-up, a caching allocator
 * that hands out every device byte), where a hidden allocation can fail or
 * fragment memory the caller has promised elsewhere.  swq_gemm_noalloc
 * computes what swq_gemm computes and allocates nothing: the fp16 copy of X
 * lives in a fixed device array inside libswq of SWQ_GEMM_NOALLOC_MAX_X_ELEMS
 * halves (16 MiB), its row scales in a second one of
 * SWQ_GEMM_NOALLOC_MAX_X_ELEMS / 32 floats (1 MiB), and the split-K partial
 * products of calls with few output tiles (small M and N) in a third of 4 Mi
 * floats (16 MiB) with 4096 tile counters -- a call whose split does not fit
 * there runs unsplit -- which every GPU that loads the library holds until
 * the process exits.  The caller passes W, X and Y as for swq_gemm.
 *   - M * K above SWQ_GEMM_NOALLOC_MAX_X_ELEMS: SWQ_ERR_BAD_SHAPE.
 *   - The first call on a device looks up the array's address on that device
 *     (cudaGetSymbolAddress with the device current); make that first call
 *     before any stream capture.
 *   - All calls on a device share the one array, which keeps the last call's
 *     contents.  Calls whose kernels overlap on the GPU (other streams, other
 *     host threads) race on it: order them on one stream or with events.
 *     Every call writes all of the array it reads, so nothing needs clearing. */
#define SWQ_GEMM_NOALLOC_MAX_X_ELEMS 8388608
swq_status swq_gemm_noalloc(int ggml_type, const void* W, const float* X, float* Y,
                            int M, int N, int K, swq_stream_t stream);

/* Options (process-wide). */
enum {
    /* 1 (default): Q2_K matmuls (GEMV, GEMM, grouped) use the activation
     * order of the reference's fused CPU routine cpu_matmul_transposed_q2_k
     * (src/tensor.h:935-945), which reads x[n + l] / x[n + l + 16] for all
     * four 2-bit planes of each 128-element half -- what
     * Compute::matmul_transposed_q returns on the reference's CPU backend, the
     * one that builds.  0: Q2_K uses the element order of dequantize_q2_k
     * (src/tensor.h:232-265), the GGUF format order, which is what the
     * reference's CUDA backend would compute (host dequantize, then SGEMM,
     * src/tensor.h:1219-1223).  swq_dequant always uses the format order. */
    SWQ_OPT_Q2K_REFERENCE_CPU_ORDER = 1,
    /* 1 (default): the GEMV and tensor-core GEMM kernels start streaming
     * weight blocks before the previous kernel on the stream has finished
     * (programmatic dependent launch); weights must then not be written by
     * the kernel immediately preceding the call.  Activations are always read
     * after that kernel completes.  0: every read waits for the preceding
     * kernel. */
    SWQ_OPT_EARLY_WEIGHT_PREFETCH = 2,
    /* Largest number of activation rows one GEMV kernel launch serves
     * (default 8); GEMV work on more rows runs in groups of this size. */
    SWQ_OPT_GEMV_MAX_M = 3,
    /* 1 (default): M >= SWQ_OPT_TENSOR_CORE_MIN_M runs the tensor-core
     * (tcgen05) dequant-GEMM, which rounds dequantized weights and
     * activations to fp16 before an fp32-accumulated product.  0: the GEMV
     * kernel over groups of rows instead.  The GEMM needs the weight base
     * 2-byte aligned; other pointers use the GEMV path. */
    SWQ_OPT_TENSOR_CORE_GEMM = 4,
    /* Smallest M that runs the tensor-core GEMM (default 5, at least 2).  The
     * GEMV kernel's cost grows with its rows (it is bound by the integer dot
     * products from about 4 rows on), so from 5 rows on the tensor cores win
     * on the Llama projection shapes. */
    SWQ_OPT_TENSOR_CORE_MIN_M = 5,
    /* Shared memory one GEMV CTA may use, in KB (0, the default: automatic --
     * half an SM, so the next kernel's CTAs fit beside this one's and start
     * streaming their weights early, unless the matrix is large enough that a
     * deeper weight ring pays more; larger values are capped at the per-block
     * maximum). */
    SWQ_OPT_GEMV_SMEM_KB = 6,
    /* Largest weight stage of the GEMV ring, in KB (0, the default: 96). */
    SWQ_OPT_GEMV_STAGE_KB = 7,
    /* GEMV CTAs per SM (0, the default: automatic; 1..4 forces it).  More
     * than one puts more consumer warps on each SM, each CTA with its share
     * of the SM's shared memory (the Q4_K tensor-core form runs 3 or 4 with
     * CTAs of 8 consumer warps instead of 16: more independent GEMVs in
     * flight at once, a longer single GEMV). */
    SWQ_OPT_GEMV_CTAS_PER_SM = 8,
    /* 1 (default): the GEMV kernel keeps the activations in fp32, as the
     * reference does: each quant value becomes an exact float and the dot
     * products are fp32 fused multiply-adds (up to 4 activation rows whose
     * fp32 copy fits the kernel's shared memory; others take the 16-bit
     * form).  0: activations rounded to 16-bit fixed point per 32-element
     * block and integer dot products (dp2a), the earlier form. */
    SWQ_OPT_GEMV_FP32_ACT = 9,
    /* Single-row GEMVs whose sub-block dot products are computed exactly in
     * integers on the tensor cores: quant values are exact small integers, x
     * is held as a 30-bit fixed-point number (four 8-bit limbs), the integer
     * sums are scaled and summed in fp32.  2 (default): Q4_K and Q6_K with x
     * in fixed point per 256-element super-block and the sub-block scales
     * applied in integers, one conversion per super-block (Q4_K: K a multiple
     * of 512 up to 8192; Q6_K: of 2048 up to 16384; activation prologues
     * included); 1: Q6_K only, in the earlier form (fixed point per
     * 16-element sub-block, one conversion per sub-block); 0: neither (the
     * fp32 form of SWQ_OPT_GEMV_FP32_ACT). */
    SWQ_OPT_GEMV_INT_MMA = 10,
    /* Largest M served by the batched K-quant GEMV: Q4_K and Q6_K with
     * 2 <= M <= this value (at most 32; K a multiple of 256, Q6_K of 2048)
     * read each weight once for all rows; per row, x is split into two fp16
     * parts relative to each 256-element super-block's largest element (22
     * bits), every product with a quant value is exact on the tensor cores
     * and the sums are fp32.  It takes precedence over the tensor-core GEMM
     * and the CUDA-core GEMV for those calls.  Default 16 (from 17 rows on,
     * the tensor-core GEMM is faster on large matrices); 0 or 1 turns it
     * off.  Its
     * scratch comes from the workspace (swq_gemm_act_ws /
     * swq_gemm_workspace_bytes) or libswq's stream-ordered pool; calls with
     * SWQ_GEMM_NOALLOC keep the tensor-core GEMM. */
    SWQ_OPT_GEMV_BATCH_MAX_M = 11,
    /* Tuning of the batched K-quant GEMV: shared-memory KB of the activation
     * table of one K split (8..160, or 0 = automatic, the default: 72, or
     * 144 for 9..16 rows on matrices that give every CTA 8 or more 16-row
     * tiles; K is split so that a split's table fits), and consumer warps per
     * 16-row tile (0 = automatic, or 1, 2, 4, 8, 16). */
    SWQ_OPT_GEMV_BATCH_TABLE_KB = 12,
    SWQ_OPT_GEMV_BATCH_GROUP = 13,
    /* Causal attention of swq_attention_prefill for head_dim 64 and 128:
     * 3 (default) on the tensor cores, q, k, v and the softmax weights as
     * pairs of fp16 numbers (22 bits relative to each q / k row's largest
     * element; v unscaled, so values far below 1 keep fewer bits: about
     * 1.7e-8 / |v| relative; exact products, fp32 sums), the context's K/V converted once
     * per call into scratch from libswq's stream-ordered pool; 2 the same
     * arithmetic converting each K/V tile in every query tile (no scratch);
     * 1 the fp32 tiled CUDA-core form; 0 one warp per row and head (the form
     * other head dims use). */
    SWQ_OPT_PREFILL_ATTENTION = 14
};
swq_status swq_set_option(int option, int value);
int swq_get_option(int option);

/* Synchronize `stream`, then read and clear the device-side status word that
 * bounded waits set on timeout.  Returns SWQ_ERR_TIMEOUT if any kernel on
 * this device gave up a wait since the last check, SWQ_ERR_CUDA if the
 * synchronize failed, else SWQ_OK. */
swq_status swq_check(swq_stream_t stream);

/* ---- Tensor-parallel all-reduce over peer memory -------------------------
 *
 * No counterpart in the reference: it runs one process, with no tensor
 * parallelism (its model forward, src/model.h:257-543, has no collective).
 * For the tensor-parallel decode of this library (one process per GPU,
 * row-parallel o and down projections), the partial products are summed with
 * a one-shot all-reduce: every rank's buffer is mapped by every other rank
 * (CUDA IPC); each call copies the rank's vector into its buffer, publishes
 * an epoch, waits (bounded) for the same slice of every peer, and sums the
 * slices in rank order, so every rank ends with the same bits.
 *   1. swq_allreduce_create on every rank (device current), for vectors of at
 *      most max_elems floats; handle_out receives SWQ_ALLREDUCE_HANDLE_BYTES
 *      bytes.
 *   2. Exchange the handles (e.g. an all-gather of bytes), then
 *      swq_allreduce_open with the world handles in rank order.
 *   3. swq_allreduce_sum(ar, data, n, stream): in place, the same n on every
 *      rank, calls in the same order on every rank (also inside CUDA graphs).
 *      A wait that gives up (a peer that never arrives) records
 *      SWQ_ERR_TIMEOUT for swq_check.
 *   4. swq_allreduce_destroy once no call is in flight on any rank.
 * After a timeout the ranks' epoch counters disagree (a rank that skipped a
 * call is one behind); swq_allreduce_reset brings the group back:
 *   a. every rank: wait until none of its sums is in flight (swq_check on the
 *      streams that ran them), then a host barrier over the group;
 *   b. every rank: swq_allreduce_reset(ar, stream) -- zeroes this rank's own
 *      flag words and epoch counters and synchronizes `stream`;
 *   c. a second host barrier; the next matched call then sums exactly.
 * Skipping barrier (c) lets a fast rank read a slow rank's stale flags.
 * At most 8 ranks. */
#define SWQ_ALLREDUCE_HANDLE_BYTES 64
typedef struct swq_allreduce swq_allreduce;
swq_status swq_allreduce_create(size_t max_elems, int rank, int world, swq_allreduce** out, void* handle_out);
swq_status swq_allreduce_open(swq_allreduce* ar, const void* handles);
swq_status swq_allreduce_sum(swq_allreduce* ar, float* data, size_t n, swq_stream_t stream);
swq_status swq_allreduce_reset(swq_allreduce* ar, swq_stream_t stream);
swq_status swq_allreduce_destroy(swq_allreduce* ar);

/* ---- MoE routing, token sort and combine ---------------------------------
 *
 * No counterpart in the reference: it has no MoE forward (its FFN is dense,
 * src/model.h:520-528; the GGUF expert tensor names appear only at
 * src/hf_loader.h:474-493).  These run the routing around the grouped expert
 * GEMMs on the device, with no count going back to the host (so a whole MoE
 * layer can be captured in a CUDA graph).  All buffers are device memory.
 *
 * swq_moe_router: logits[t][e] = router_w[e] . X[t] (fp32, router_w E x H,
 *   X T x H), then per token the k largest logits in descending order (ties:
 *   the lower expert id first; NaN ranks as -inf) into topk_ids [T][k], and
 *   topk_w [T][k] = softmax over those k logits (exp(l_j - l_0) / sum_i
 *   exp(l_i - l_0), the sum left to right).  logits [T][E] is written too.
 *   E <= SWQ_MOE_MAX_EXPERTS, k <= min(E, SWQ_MOE_MAX_TOPK); one token row
 *   (H floats) must fit the shared memory of a CTA.
 * swq_moe_sort: the P = T*k pairs p = t*k + j of topk_ids, stably sorted by
 *   expert: expert_offsets [n_experts + 1] (expert e's rows are
 *   expert_offsets[e] .. expert_offsets[e+1]-1), sorted_pairs [P] (the pair of
 *   each row) and pair_rows [P] (the row of each pair).  A pair whose id is
 *   outside [0, n_experts) gets row -1 and no row, and swq_check then returns
 *   SWQ_ERR_BAD_ARG.
 * swq_moe_gather: X_sorted[r] = X[sorted_pairs[r] / k] for the rows
 *   r < expert_offsets[n_experts] (H floats each): the input of
 *   swq_grouped_gemm / swq_grouped_gemv.
 * swq_moe_combine: Y[t] = (accumulate ? Y[t] : 0) + sum_j topk_w[t][j] *
 *   Y_sorted[pair_rows[t*k + j]], one fused multiply-add per slot in the
 *   order j = 0 .. k-1 (rows -1 add nothing). */
#define SWQ_MOE_MAX_EXPERTS 1024
#define SWQ_MOE_MAX_TOPK 32
swq_status swq_moe_router(const float* router_w, const float* X, int T, int E, int H, int k, float* logits,
                          int* topk_ids, float* topk_w, swq_stream_t stream);
swq_status swq_moe_sort(const int* topk_ids, int P, int n_experts, int* expert_offsets, int* sorted_pairs,
                        int* pair_rows, swq_stream_t stream);
swq_status swq_moe_gather(const float* X, const int* sorted_pairs, const int* expert_offsets, int n_experts, int P,
                          int k, int H, float* X_sorted, swq_stream_t stream);
swq_status swq_moe_combine(const float* Y_sorted, const int* pair_rows, const float* topk_w, int T, int k, int H,
                           float* Y, int accumulate, swq_stream_t stream);

/* ---- Expert-parallel dispatch and combine over peer memory ---------------
 *
 * No counterpart in the reference (see above).  The experts of a MoE layer
 * are sharded over the `world` GPUs of a group (one process per GPU; rank r
 * owns experts r*E/world .. (r+1)*E/world - 1).  Each rank's token rows
 * travel to the ranks that own their experts by peer stores over NVLink
 * (CUDA IPC), with the per-expert counts exchanged on the device, so nothing
 * returns to the host; every wait is bounded (1 s) and records
 * SWQ_ERR_TIMEOUT for swq_check.
 *   1. swq_ep_create on every rank (device current): at most max_tokens tokens
 *      per call, top_k slots each, n_experts (a multiple of world), hidden H.
 *      handle_out receives SWQ_EP_HANDLE_BYTES bytes.  Device memory:
 *      (world + 1) * max_tokens * top_k rows of H floats, plus small tables.
 *   2. Exchange the handles, then swq_ep_open with all of them in rank order.
 *   3. Per MoE layer, on every rank, in the same order:
 *      swq_ep_dispatch(X [T][H], topk_ids [T][k] global expert ids, T);
 *      swq_ep_received gives the rows this rank received (X_recv, capacity
 *      rows of H floats) and their device expert offsets (E/world + 1 ints,
 *      this rank's experts in order; rows beyond the last offset are
 *      unused): the input of swq_grouped_gemm / swq_grouped_gemv with
 *      total_rows = capacity;
 *      swq_ep_combine(Y_recv, topk_w, Y): Y_recv holds the expert outputs of
 *      the received rows (capacity x H, same row order); Y [T][H] receives
 *      (accumulate ? Y : 0) + sum_j topk_w[t][j] * output of pair (t, j), one
 *      fused multiply-add per slot in the order j = 0 .. k-1.
 *   4. After a timeout: every rank waits until none of its calls is in
 *      flight, meets the others at a host barrier, calls swq_ep_reset, and
 *      meets them again (as for swq_allreduce_reset).
 *   5. swq_ep_destroy once no call is in flight on any rank.
 * With world = 1 the same calls run on one GPU without IPC peers.  At most
 * SWQ_EP_MAX_RANKS ranks. */
#define SWQ_EP_MAX_RANKS 8
#define SWQ_EP_HANDLE_BYTES 64
typedef struct swq_ep swq_ep;
swq_status swq_ep_create(int max_tokens, int top_k, int n_experts, int hidden, int rank, int world, swq_ep** out,
                         void* handle_out);
swq_status swq_ep_open(swq_ep* ep, const void* handles);
swq_status swq_ep_dispatch(swq_ep* ep, const float* X, const int* topk_ids, int T, swq_stream_t stream);
swq_status swq_ep_received(const swq_ep* ep, float** X_recv, const int** expert_offsets, int* capacity);
swq_status swq_ep_combine(swq_ep* ep, const float* Y_recv, const float* topk_w, float* Y, int accumulate,
                          swq_stream_t stream);
swq_status swq_ep_reset(swq_ep* ep, swq_stream_t stream);
swq_status swq_ep_destroy(swq_ep* ep);

/* ---- Host-buffer entry point (the reference's calling convention) --------
 *
 * Mirrors Compute::matmul_transposed_q(out, x, QuantWeight{data,type}, N, K)
 * (src/tensor.h:1212) with host fp32 `out`/`x` and a host pointer to the GGUF
 * blocks, as Model::forward calls it (src/model.h:284-539).  The blocks are
 * uploaded to the device once per (pointer, type, N, K) and stay resident,
 * like the reference's GPUWeightCache keyed by host pointer
 * (src/cuda_kernels.cu:88-127), but the key includes the shape so that a
 * reused host address of a different matrix never aliases.  Blocks must stay
 * unchanged while cached; swq_ctx_evict drops one entry.  Synchronous: returns
 * when `out` holds the result. */
typedef struct swq_ctx* swq_ctx_t;
swq_status swq_ctx_create(int device, swq_ctx_t* ctx);
swq_status swq_ctx_destroy(swq_ctx_t ctx);
swq_status swq_ctx_matmul_transposed_q(swq_ctx_t ctx, float* out, const float* x,
                                       const void* w_host, int ggml_type, int N, int K);
/* Same for M activation rows (X: M x K, Y: M x N, host, row-major). */
swq_status swq_ctx_matmul_q_batched(swq_ctx_t ctx, float* Y, const float* X,
                                    const void* w_host, int ggml_type, int M, int N, int K);
/* dequantize() with host src/dst (src/tensor.h:451). */
swq_status swq_ctx_dequantize(swq_ctx_t ctx, const void* src_host, float* dst_host,
                              int64_t n, int ggml_type);
swq_status swq_ctx_evict(swq_ctx_t ctx, const void* w_host);
/* Bytes of weight blocks currently resident for this context. */
size_t swq_ctx_resident_bytes(swq_ctx_t ctx);

#ifdef __cplusplus
}
#endif

#endif /* SWQ_H */
