/* moe_oracle.c -- CPU restatement of the MoE routing, sort and combine
 * (TEST INFRASTRUCTURE ONLY; linked into liboracle.so).
 *
 * The reference has no MoE forward (src/model.h:520-528 is a dense FFN; the
 * GGUF expert names appear only at src/hf_loader.h:474-493), so nothing here
 * restates reference code: these functions state the routing of the MoE
 * decoder shape (fp32 router, the top-k logits, softmax over those k, tokens
 * grouped by expert, weighted sum of the expert outputs) in plain C, the way
 * libswq's kernels define it, for the parity tests.  Parity for routing is
 * unpinned by the reference.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* logits[t][e] = sum_h W[e][h] * X[t][h], in double (the GPU sums in fp32 in
 * another order: compare with a tolerance). */
void oracle_moe_router_logits(const float* W, const float* X, int T, int E, int H, double* out) {
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < E; ++e) {
            double acc = 0.0;
            for (int h = 0; h < H; ++h) acc += (double)W[(int64_t)e * H + h] * (double)X[(int64_t)t * H + h];
            out[(int64_t)t * E + e] = acc;
        }
}

/* Per token: the k largest logits in descending order, ties broken by the
 * lower expert id, NaN counted as -inf; w_j = expf(l_j - l_0) / sum, the sum
 * of the k exponentials taken left to right in float. */
void oracle_moe_topk_softmax(const float* logits, int T, int E, int k, int* ids, float* w) {
    unsigned char taken[4096];
    for (int t = 0; t < T; ++t) {
        const float* l = logits + (int64_t)t * E;
        memset(taken, 0, (size_t)E);
        float v[64];
        for (int j = 0; j < k; ++j) {
            float bv = -INFINITY;
            int bi = -1;
            for (int e = 0; e < E; ++e) {
                if (taken[e]) continue;
                float x = l[e];
                if (x != x) x = -INFINITY;
                if (bi < 0 || x > bv) {
                    bv = x;
                    bi = e;
                }
            }
            taken[bi] = 1;
            ids[(int64_t)t * k + j] = bi;
            v[j] = bv;
        }
        float ex[64], sum = 0.f;
        for (int j = 0; j < k; ++j) {
            ex[j] = expf(v[j] - v[0]);
            sum += ex[j];
        }
        for (int j = 0; j < k; ++j) w[(int64_t)t * k + j] = ex[j] / sum;
    }
}

/* Stable counting sort of the P pairs by expert id: offsets[E+1], sorted[rows]
 * (pair of each row), prow[P] (row of each pair, -1 for an id outside
 * [0, E)).  Returns the number of pairs left out. */
int oracle_moe_sort(const int* ids, int P, int E, int* offsets, int* sorted, int* prow) {
    int bad = 0;
    for (int e = 0; e <= E; ++e) offsets[e] = 0;
    for (int p = 0; p < P; ++p) {
        if (ids[p] >= 0 && ids[p] < E) offsets[ids[p] + 1]++;
        else bad++;
    }
    for (int e = 0; e < E; ++e) offsets[e + 1] += offsets[e];
    int fill[4096];
    for (int e = 0; e < E; ++e) fill[e] = offsets[e];
    for (int p = 0; p < P; ++p) {
        const int e = ids[p];
        if (e >= 0 && e < E) {
            prow[p] = fill[e];
            sorted[fill[e]++] = p;
        } else {
            prow[p] = -1;
        }
    }
    return bad;
}

/* Y[t][h] = (accumulate ? Y[t][h] : 0) + sum_j w[t][j] * Ys[prow[t*k+j]][h],
 * one fmaf per slot, j = 0 .. k-1; rows -1 add nothing. */
void oracle_moe_combine(const float* Ys, const int* prow, const float* w, int T, int k, int H, float* Y,
                        int accumulate) {
    for (int t = 0; t < T; ++t)
        for (int h = 0; h < H; ++h) {
            float acc = accumulate ? Y[(int64_t)t * H + h] : 0.f;
            for (int j = 0; j < k; ++j) {
                const int r = prow[t * k + j];
                if (r >= 0) acc = fmaf(w[t * k + j], Ys[(int64_t)r * H + h], acc);
            }
            Y[(int64_t)t * H + h] = acc;
        }
}
