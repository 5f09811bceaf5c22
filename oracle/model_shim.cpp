// model_shim.cpp -- C ABI over the reference's GGUF reader and dense model
// forward (src/gguf.h, src/model.h), compiled from the reference sources where
// they lie (see oracle/Makefile).  TEST INFRASTRUCTURE ONLY: it pins the CPU
// restatement of the decode forward (oracle/model_ref.py) and libswq's GGUF
// reader (swq/gguf.py) against the reference's own code.  Never part of libswq.
//
//   refg_*  -> GGUFFile::load / parse / get_* / tensors   src/gguf.h:224-419
//   refm_*  -> Model::load / forward / clear_state       src/model.h:213-543
//              (Backend::CPU: the fused per-format CPU matmuls)
#include <cstdint>
#include <cstring>
#include <string>

#include "model.h"

// Backend the refm_* entry points load the model with: the CPU build, or
// Backend::CUDA in the drop-in build (make_dropin.py, dropin_backend.cpp).
#ifndef REF_BACKEND
#define REF_BACKEND Backend::CPU
#endif

extern "C" {

// ---- GGUF file ----

void* refg_open(const char* path) {
    auto* g = new GGUFFile();
    if (!g->load(path)) {
        delete g;
        return nullptr;
    }
    return g;
}

void refg_close(void* h) { delete static_cast<GGUFFile*>(h); }

// version, tensor_count, metadata_kv_count, alignment, data_offset
void refg_header(void* h, unsigned long long out[5]) {
    const auto* g = static_cast<const GGUFFile*>(h);
    out[0] = g->version;
    out[1] = g->tensor_count;
    out[2] = g->metadata_kv_count;
    out[3] = g->alignment;
    out[4] = g->data_offset;
}

// 1 if found: type, n_dims, dims[4], offset, num_bytes
int refg_tensor(void* h, const char* name, unsigned* type, unsigned* n_dims, unsigned long long dims[4],
                unsigned long long* offset, unsigned long long* num_bytes) {
    const auto* g = static_cast<const GGUFFile*>(h);
    auto it = g->tensors.find(name);
    if (it == g->tensors.end()) return 0;
    const GGUFTensorInfo& t = it->second;
    *type = static_cast<unsigned>(t.type);
    *n_dims = t.n_dims;
    for (int d = 0; d < 4; ++d) dims[d] = t.dims[d];
    *offset = t.offset;
    *num_bytes = t.num_bytes();
    return 1;
}

// Byte offset of the tensor's data from the start of the file (-1: absent).
long long refg_tensor_file_offset(void* h, const char* name) {
    const auto* g = static_cast<const GGUFFile*>(h);
    const void* p = g->get_tensor_data(name);
    if (!p) return -1;
    return static_cast<const uint8_t*>(p) - g->file_data;
}

long long refg_get_i64(void* h, const char* key, long long def) {
    return static_cast<GGUFFile*>(h)->get_i64(key, def);
}

double refg_get_f64(void* h, const char* key, double def) { return static_cast<GGUFFile*>(h)->get_f64(key, def); }

// Copies the string value (truncated to cap-1 bytes); returns its full length.
long long refg_get_str(void* h, const char* key, char* out, long long cap) {
    const std::string s = static_cast<GGUFFile*>(h)->get_str(key, "");
    if (cap > 0) {
        const size_t n = s.size() < static_cast<size_t>(cap - 1) ? s.size() : static_cast<size_t>(cap - 1);
        memcpy(out, s.data(), n);
        out[n] = '\0';
    }
    return static_cast<long long>(s.size());
}

// Array length of the value under key (-1: absent or not an array).
long long refg_array_len(void* h, const char* key) {
    const auto* g = static_cast<const GGUFFile*>(h);
    auto it = g->metadata.find(key);
    if (it == g->metadata.end() || it->second.type != GGUF_TYPE_ARRAY) return -1;
    return static_cast<long long>(it->second.arr.size());
}

// ---- model ----

void* refm_load(const char* path, int context_override) {
    auto* m = new Model(REF_BACKEND);
    if (!m->load(path, context_override)) {
        delete m;
        return nullptr;
    }
    return m;
}

void refm_free(void* h) { delete static_cast<Model*>(h); }

// hidden, ffn, layers, heads, kv_heads, head_dim, vocab, max_seq, rope_neox, rope_dim
void refm_config_i(void* h, int out[10]) {
    const ModelConfig& c = static_cast<Model*>(h)->config;
    out[0] = c.hidden_size;
    out[1] = c.intermediate_size;
    out[2] = c.num_layers;
    out[3] = c.num_heads;
    out[4] = c.num_kv_heads;
    out[5] = c.head_dim;
    out[6] = c.vocab_size;
    out[7] = c.max_seq_len;
    out[8] = c.rope_neox ? 1 : 0;
    out[9] = c.rope_dim;
}

// rms_norm_eps, rope_theta
void refm_config_f(void* h, float out[2]) {
    const ModelConfig& c = static_cast<Model*>(h)->config;
    out[0] = c.rms_norm_eps;
    out[1] = c.rope_theta;
}

// Logits of `token` at `pos` (vocab floats copied to out).
void refm_forward(void* h, int token, int pos, float* out) {
    auto* m = static_cast<Model*>(h);
    const float* l = m->forward(token, pos);
    memcpy(out, l, sizeof(float) * static_cast<size_t>(m->config.vocab_size));
}

void refm_clear(void* h) { static_cast<Model*>(h)->clear_state(); }

}  // extern "C"
